// CKL B200 runtime: devices, buffers, bound plans, graph executor and the C ABI.
//
// The structure follows the reference executor (lib/Runtime/NvidiaProgram.cpp and
// lib/Runtime/NvidiaRuntime.cpp): a program's packed entry runs once per bind and builds a
// bound plan through eight callbacks; the plan then replays as ordinary launches, a
// single-stream capture or an explicit CUDA graph whose edges are the inferred dependencies.
// The B200 build uses the CUDA runtime API (linked statically, so the library loads on
// machines without a driver), resolves kernel names against the linked sm_100a library or a
// loaded CUBIN, and adds asynchronous submission and host-copy entry points.
#include "ckl_b200.h"
#include "errors.hpp"
#include "library.hpp"
#include "planner.hpp"

#include <cuda_profiler_api.h>
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <thread>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

thread_local std::string lastError;

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void check(cudaError_t status, const char *operation) {
  if (status != cudaSuccess) {
    cudaGetLastError();
    throw CudaError(std::string(operation) + " failed: " + cudaGetErrorName(status) + ": " +
                    cudaGetErrorString(status));
  }
}

template <typename F> int guarded(F &&body) {
  try {
    body();
    return CKL_OK;
  } catch (const std::invalid_argument &e) {
    lastError = e.what();
    return CKL_INVALID_ARGUMENT;
  } catch (const std::out_of_range &e) {
    lastError = e.what();
    return CKL_OUT_OF_RANGE;
  } catch (const std::exception &e) {
    lastError = e.what();
    return CKL_RUNTIME_ERROR;
  } catch (...) {
    lastError = "unknown native failure";
    return CKL_RUNTIME_ERROR;
  }
}

} // namespace

void ckl::setLastError(const std::string &message) { lastError = message; }

namespace {

std::atomic<uint64_t> nextDeviceId{0};
constexpr const char kLibraryMarker[] = "ckl-b200:library";

struct Device {
  int ordinal = 0;
  uint64_t id = 0;
  std::string name;
  // Set before asynchronous work is enqueued on this device (ckl_launch, asynchronous
  // copies); a synchronous buffer copy then waits for the device first, so it never races
  // with a submission still in flight.
  mutable std::atomic<bool> asyncPending{false};
  void current() const { check(cudaSetDevice(ordinal), "cudaSetDevice"); }
  void settle() const {
    if (asyncPending.exchange(false))
      check(cudaDeviceSynchronize(), "cudaDeviceSynchronize(settle)");
  }
};

struct Allocation {
  std::shared_ptr<Device> device;
  uint64_t pointer = 0;
  std::size_t bytes = 0;
  bool owned = true;
  ~Allocation() {
    if (owned && pointer) {
      cudaSetDevice(device->ordinal);
      cudaFree(reinterpret_cast<void *>(pointer));
    }
  }
};

struct Module {
  std::shared_ptr<Device> device;
  bool library = true;
  cudaLibrary_t handle = nullptr;
  ~Module() {
    if (handle) {
      cudaSetDevice(device->ordinal);
      cudaLibraryUnload(handle);
    }
  }
};

struct Function {
  const void *address = nullptr;
  const ckl::library::Kernel *entry = nullptr; // library kernels only
  std::shared_ptr<Module> module;
  std::string name;
};

struct KernelLaunch {
  Function function;
  dim3 grid, block;
  unsigned shared = 0;
  std::vector<std::vector<unsigned char>> arguments;
  std::vector<void *> pointers() const {
    std::vector<void *> out;
    out.reserve(arguments.size());
    for (const auto &a : arguments)
      out.push_back(const_cast<unsigned char *>(a.data()));
    return out;
  }
};

struct Plan {
  std::vector<KernelLaunch> nodes;
  std::vector<std::vector<std::size_t>> dependencies;
  std::size_t add(KernelLaunch launch, std::vector<std::size_t> deps) {
    if (!launch.function.address)
      throw std::invalid_argument("kernel plan node requires a resolved function");
    std::size_t id = nodes.size();
    for (std::size_t d : deps)
      if (d >= id)
        throw std::invalid_argument("kernel dependencies must reference earlier plan nodes");
    nodes.push_back(std::move(launch));
    dependencies.push_back(std::move(deps));
    return id;
  }
  Plan repeat(std::size_t iterations) const {
    Plan out;
    auto deps = ckl::planning::repeatDependencies(dependencies, iterations);
    for (std::size_t i = 0; i < deps.size(); ++i)
      out.add(nodes[i % nodes.size()], std::move(deps[i]));
    return out;
  }
};

struct GraphExec {
  std::shared_ptr<Device> device;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<cudaGraphNode_t> nodes;
  std::vector<KernelLaunch> launches; // explicit graphs: the launch behind each node
  bool captured = false;
  ~GraphExec() {
    cudaSetDevice(device->ordinal);
    if (exec)
      cudaGraphExecDestroy(exec);
    if (graph)
      cudaGraphDestroy(graph);
  }
};

// Programmatic dependent launch for library kernels that wait on their predecessors
// themselves (griddepcontrol.wait at entry): such a kernel is scheduled while the kernel before
// it finishes, hiding most of the launch gap between dependent nodes.  CKL_B200_DEPENDENT_LAUNCH=0
// turns it off (every edge then waits for full completion); CKL_B200_DEPENDENT_LAUNCH_EXCLUDE
// lists comma-separated kernel-name fragments to leave out (tuning).
bool dependentLaunch(const KernelLaunch &k) {
  static const bool enabled = [] {
    const char *value = std::getenv("CKL_B200_DEPENDENT_LAUNCH");
    return !(value && value[0] == '0');
  }();
  static const std::vector<std::string> excluded = [] {
    std::vector<std::string> out;
    if (const char *value = std::getenv("CKL_B200_DEPENDENT_LAUNCH_EXCLUDE")) {
      std::string list(value);
      for (std::size_t start = 0; start <= list.size();) {
        const std::size_t end = std::min(list.find(',', start), list.size());
        if (end > start)
          out.push_back(list.substr(start, end - start));
        start = end + 1;
      }
    }
    return out;
  }();
  if (!enabled || !k.function.entry || !k.function.entry->dependentLaunch)
    return false;
  for (const std::string &fragment : excluded)
    if (std::strstr(k.function.entry->name, fragment.c_str()))
      return false;
  return true;
}

void launchOne(const KernelLaunch &k, cudaStream_t stream) {
  auto args = k.pointers();
  if (!dependentLaunch(k)) {
    check(cudaLaunchKernel(k.function.address, k.grid, k.block, args.data(), k.shared, stream),
          "cudaLaunchKernel");
    return;
  }
  cudaLaunchConfig_t config{};
  config.gridDim = k.grid;
  config.blockDim = k.block;
  config.dynamicSmemBytes = k.shared;
  config.stream = stream;
  cudaLaunchAttribute attribute{};
  attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute.val.programmaticStreamSerializationAllowed = 1;
  config.attrs = &attribute;
  config.numAttrs = 1;
  check(cudaLaunchKernelExC(&config, k.function.address, args.data()), "cudaLaunchKernelEx");
}

void launchOrdinary(const Plan &plan, cudaStream_t stream) {
  for (const KernelLaunch &k : plan.nodes)
    launchOne(k, stream);
}

std::shared_ptr<GraphExec> instantiate(const Plan &plan, const std::shared_ptr<Device> &device) {
  if (plan.nodes.empty())
    throw std::invalid_argument("cannot instantiate an empty plan");
  auto g = std::make_shared<GraphExec>();
  g->device = device;
  check(cudaGraphCreate(&g->graph, 0), "cudaGraphCreate");
  g->nodes.reserve(plan.nodes.size());
  for (std::size_t i = 0; i < plan.nodes.size(); ++i) {
    const KernelLaunch &k = plan.nodes[i];
    auto args = k.pointers();
    cudaKernelNodeParams p{};
    p.func = const_cast<void *>(k.function.address);
    p.gridDim = k.grid;
    p.blockDim = k.block;
    p.sharedMemBytes = k.shared;
    p.kernelParams = args.data();
    cudaGraphNode_t node{};
    check(cudaGraphAddKernelNode(&node, g->graph, nullptr, 0, &p), "cudaGraphAddKernelNode");
    g->nodes.push_back(node);
    // Edges into a dependent-launch-aware kernel are programmatic: it may start once every
    // predecessor has triggered (griddepcontrol.launch_dependents) and waits for their
    // completion itself.
    const bool programmatic = dependentLaunch(k);
    for (std::size_t d : plan.dependencies[i]) {
      cudaGraphEdgeData edge{};
      if (programmatic) {
        edge.from_port = cudaGraphKernelNodePortProgrammatic;
        edge.type = cudaGraphDependencyTypeProgrammatic;
      }
      const cudaGraphNode_t from = g->nodes.at(d);
      check(cudaGraphAddDependencies_v2(g->graph, &from, &node, &edge, 1),
            "cudaGraphAddDependencies");
    }
  }
  check(cudaGraphInstantiate(&g->exec, g->graph, 0), "cudaGraphInstantiate");
  g->launches = plan.nodes;
  return g;
}

std::shared_ptr<GraphExec> capture(const Plan &plan, cudaStream_t stream,
                                   const std::shared_ptr<Device> &device) {
  if (plan.nodes.empty())
    throw std::invalid_argument("capture requires a nonempty plan");
  auto g = std::make_shared<GraphExec>();
  g->device = device;
  g->captured = true;
  check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  try {
    launchOrdinary(plan, stream);
  } catch (...) {
    cudaGraph_t abandoned = nullptr;
    cudaStreamEndCapture(stream, &abandoned);
    if (abandoned)
      cudaGraphDestroy(abandoned);
    throw;
  }
  check(cudaStreamEndCapture(stream, &g->graph), "cudaStreamEndCapture");
  std::size_t count = 0;
  check(cudaGraphGetNodes(g->graph, nullptr, &count), "cudaGraphGetNodes");
  g->nodes.resize(count);
  check(cudaGraphGetNodes(g->graph, g->nodes.data(), &count), "cudaGraphGetNodes");
  check(cudaGraphInstantiate(&g->exec, g->graph, 0), "cudaGraphInstantiate(captured)");
  return g;
}

// ---- textual executable plans ----------------------------------------------------------
struct ExecArg {
  enum Kind { Resource, Scalar, Value } kind = Resource;
  uint64_t resource = 0, offset = 0;
  uint32_t argument = 0;
  std::vector<unsigned char> bytes;
};
struct ExecKernel {
  uint64_t id = 0;
  std::string name;
  uint64_t grid[3] = {1, 1, 1}, block[3] = {1, 1, 1}, shared = 0;
  std::vector<ExecArg> arguments;
  std::vector<uint64_t> dependencies;
};
struct ExecResource {
  bool external = false;
  uint32_t argument = 0;
  uint64_t heap = 0, offset = 0;
};
struct ExecPlan {
  std::vector<unsigned char> binary;
  uint64_t alignment = 1; // caller buffers must start on this boundary (else: the fallback)
  std::vector<uint64_t> heaps;
  std::vector<ExecResource> resources;
  std::vector<ExecKernel> kernels;
  std::vector<uint64_t> bufferBytes;
  std::vector<std::string> scalarTypes;
};

std::vector<unsigned char> fromHex(const std::string &hex) {
  if (hex.size() % 2)
    throw std::invalid_argument("odd hex byte string in plan");
  std::vector<unsigned char> out(hex.size() / 2);
  for (std::size_t i = 0; i < out.size(); ++i)
    out[i] = static_cast<unsigned char>(std::stoul(hex.substr(2 * i, 2), nullptr, 16));
  return out;
}

std::shared_ptr<ExecPlan> parsePlan(const char *text) {
  if (!text)
    throw std::invalid_argument("plan text is null");
  auto plan = std::make_shared<ExecPlan>();
  std::istringstream input(text);
  std::string line;
  bool header = false, ended = false;
  while (std::getline(input, line)) {
    std::istringstream in(line);
    std::string op;
    if (!(in >> op) || op[0] == '#')
      continue;
    if (op == "ckl-b200-plan") {
      int version = 0;
      in >> version;
      if (version != 1)
        throw std::invalid_argument("unsupported plan version");
      header = true;
    } else if (op == "arg") {
      uint32_t index;
      std::string kind, value;
      in >> index >> kind >> value;
      if (index != plan->bufferBytes.size())
        throw std::invalid_argument("plan arguments must be listed in order");
      if (kind == "buffer") {
        plan->bufferBytes.push_back(std::stoull(value));
        plan->scalarTypes.push_back("");
      } else if (kind == "scalar") {
        plan->bufferBytes.push_back(0);
        plan->scalarTypes.push_back(value);
      } else {
        throw std::invalid_argument("unknown plan argument kind: " + kind);
      }
    } else if (op == "binary") {
      std::string kind;
      in >> kind;
      if (kind == "library") {
        plan->binary.assign(kLibraryMarker, kLibraryMarker + sizeof(kLibraryMarker) - 1);
      } else if (kind == "hex") {
        std::string hex;
        in >> hex;
        plan->binary = fromHex(hex);
      } else {
        throw std::invalid_argument("unknown plan binary kind: " + kind);
      }
    } else if (op == "align") {
      in >> plan->alignment;
      if (!in.fail() && (plan->alignment == 0 || (plan->alignment & (plan->alignment - 1))))
        throw std::invalid_argument("plan alignment must be a power of two");
    } else if (op == "heap") {
      uint64_t id, bytes;
      in >> id >> bytes;
      if (id != plan->heaps.size())
        throw std::invalid_argument("plan heaps must be listed in order");
      plan->heaps.push_back(bytes);
    } else if (op == "resource") {
      uint64_t id;
      std::string kind;
      in >> id >> kind;
      if (id != plan->resources.size())
        throw std::invalid_argument("plan resources must be listed in order");
      ExecResource r;
      if (kind == "external") {
        r.external = true;
        in >> r.argument;
      } else if (kind == "temporary") {
        in >> r.heap >> r.offset;
      } else {
        throw std::invalid_argument("unknown plan resource kind: " + kind);
      }
      plan->resources.push_back(r);
    } else if (op == "kernel") {
      ExecKernel k;
      in >> k.id >> k.name >> k.grid[0] >> k.grid[1] >> k.grid[2] >> k.block[0] >> k.block[1] >>
          k.block[2] >> k.shared;
      plan->kernels.push_back(std::move(k));
    } else if (op == "argres" || op == "argscalar" || op == "argvalue" || op == "dep") {
      if (plan->kernels.empty())
        throw std::invalid_argument("plan argument outside a kernel");
      ExecKernel &k = plan->kernels.back();
      if (op == "dep") {
        uint64_t id;
        in >> id;
        k.dependencies.push_back(id);
        continue;
      }
      ExecArg a;
      if (op == "argres") {
        a.kind = ExecArg::Resource;
        in >> a.resource >> a.offset;
      } else if (op == "argscalar") {
        a.kind = ExecArg::Scalar;
        in >> a.argument;
      } else {
        a.kind = ExecArg::Value;
        std::string hex;
        in >> hex;
        a.bytes = fromHex(hex);
      }
      k.arguments.push_back(std::move(a));
    } else if (op == "end") {
      ended = true;
      break;
    } else {
      throw std::invalid_argument("unknown plan record: " + op);
    }
    if (in.fail())
      throw std::invalid_argument("malformed plan record: " + line);
  }
  if (!header || !ended)
    throw std::invalid_argument("plan text lacks its header or end record");
  if (plan->binary.empty())
    throw std::invalid_argument("plan names no device binary");
  return plan;
}

struct ProgramState {
  ckl_entry_fn entry = nullptr;
  std::vector<uint64_t> bufferBytes;
  std::vector<std::string> scalarTypes;
  std::shared_ptr<ProgramState> fallback;
  std::shared_ptr<ExecPlan> plan;
  std::mutex moduleMutex;
  std::map<uint64_t, std::shared_ptr<Module>> modules;
};

struct InvocationState {
  std::shared_ptr<ProgramState> program;
  std::shared_ptr<Device> device;
  cudaStream_t stream = nullptr;
  std::shared_ptr<Module> module;
  std::vector<std::shared_ptr<Allocation>> heaps;
  std::vector<std::shared_ptr<Allocation>> buffers; // keep bound caller storage alive
  std::vector<uint64_t> resources;
  Plan plan;
  KernelLaunch pending;
  std::vector<std::size_t> pendingDeps;
  std::map<uint64_t, std::size_t> nodes;
  std::map<std::pair<int, uint64_t>, std::shared_ptr<GraphExec>> graphs;
  std::mutex runMutex;
  std::string error;
  bool boundedWaits = false; // some node waits with bounded waits (library fault word)
  ~InvocationState() {
    graphs.clear();
    if (stream) {
      cudaSetDevice(device->ordinal);
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }
};

// The packed entry of a textual plan: the same callback sequence the reference's generated
// entry performs (lib/Transforms/ExecToLLVM.cpp:25-120).
void planEntry(void **packed) {
  void *frame = *static_cast<void **>(packed[0]);
  void **values = *static_cast<void ***>(packed[1]);
  auto *state = static_cast<InvocationState *>(frame);
  const ExecPlan &plan = *state->program->plan;
  ckl_begin(frame, plan.binary.data(), plan.binary.size());
  for (std::size_t h = 0; h < plan.heaps.size(); ++h)
    ckl_heap(frame, h, plan.heaps[h]);
  for (std::size_t r = 0; r < plan.resources.size(); ++r) {
    const ExecResource &res = plan.resources[r];
    ckl_resource(frame, r, res.external ? 0 : res.heap, res.external ? 0 : res.offset,
                 res.external ? values[res.argument] : nullptr);
  }
  for (const ExecKernel &k : plan.kernels) {
    ckl_kernel(frame, k.name.c_str(), k.grid[0], k.grid[1], k.grid[2], k.block[0], k.block[1],
               k.block[2], k.shared);
    for (const ExecArg &a : k.arguments) {
      if (a.kind == ExecArg::Resource) {
        ckl_argument_resource(frame, a.resource, a.offset);
      } else if (a.kind == ExecArg::Scalar) {
        const std::string &type = state->program->scalarTypes.at(a.argument);
        uint64_t size = (type == "i64" || type == "f64") ? 8 : 4;
        ckl_argument_value(frame, values[a.argument], size);
      } else {
        ckl_argument_value(frame, a.bytes.data(), a.bytes.size());
      }
    }
    for (uint64_t d : k.dependencies)
      ckl_dependency(frame, d);
    ckl_commit(frame, k.id);
  }
}

template <typename F> void callback(void *opaque, F &&action) {
  auto &frame = *static_cast<InvocationState *>(opaque);
  if (!frame.error.empty())
    return;
  try {
    action(frame);
  } catch (const std::exception &e) {
    frame.error = e.what();
  } catch (...) {
    frame.error = "unknown callback failure";
  }
}

void validateExecution(const InvocationState &f, int mode, uint64_t batch) {
  if (mode < 0 || mode > 2 || !batch || f.plan.nodes.empty() ||
      batch > 1000000 / f.plan.nodes.size())
    throw std::invalid_argument(
        "invalid execution mode or batch exceeds one million kernel nodes");
}

GraphExec &executionGraph(InvocationState &f, int mode, uint64_t batch) {
  auto &graph = f.graphs[{mode, batch}];
  if (!graph) {
    Plan plan = batch == 1 ? f.plan : f.plan.repeat(batch);
    graph = mode == 2 ? capture(plan, f.stream, f.device) : instantiate(plan, f.device);
  }
  return *graph;
}

void submit(InvocationState &f, int mode, uint64_t batch) {
  if (mode) {
    check(cudaGraphLaunch(executionGraph(f, mode, batch).exec, f.stream), "cudaGraphLaunch");
  } else {
    for (uint64_t i = 0; i < batch; ++i)
      launchOrdinary(f.plan, f.stream);
  }
}

// After an invocation's work has completed: a kernel with bounded waits that gave one up did
// not do its work, so the submission's results are invalid.  The fault word stays set (for
// every later check on the device) until the caller clears it with ckl_library_faults(&w, 1).
void checkLibraryFaults(const InvocationState &f) {
  if (!f.boundedWaits)
    return;
  uint32_t word = 0;
  if (ckl_library_faults(&word, 0) != CKL_OK)
    throw CudaError("reading the kernel library's fault word failed");
  if (word) {
    char text[256];
    std::snprintf(text, sizeof text,
                  "kernel library fault word 0x%x on device %d: a tensor-core kernel gave up a "
                  "bounded wait (bit 0) or found a misaligned operand (bit 1) and skipped its "
                  "work; the results are invalid (clear with ckl_library_faults(&word, 1))",
                  word, f.device->ordinal);
    throw std::runtime_error(text);
  }
}

void requireScalarType(const std::string &type, uint32_t kind) {
  static const std::map<std::string, uint32_t> kinds = {
      {"i32", CKL_ARG_I32}, {"i64", CKL_ARG_I64}, {"f32", CKL_ARG_F32}, {"f64", CKL_ARG_F64}};
  auto found = kinds.find(type);
  if (found == kinds.end())
    throw std::invalid_argument("unsupported scalar binding type");
  if (found->second != kind)
    throw std::invalid_argument("argument type does not match compiled signature");
}

} // namespace

// ---- opaque handles --------------------------------------------------------------------
struct ckl_device {
  std::shared_ptr<Device> device;
};
struct ckl_buffer {
  std::shared_ptr<Allocation> allocation;
  std::size_t offset = 0;
  std::size_t bytes = 0;
  uint64_t address() const { return allocation->pointer + offset; }
};
struct ckl_program {
  std::shared_ptr<ProgramState> state;
};
struct ckl_invocation {
  std::shared_ptr<InvocationState> state;
};
// A point on an invocation's stream.  It shares the invocation's state, so the stream, heaps
// and bound buffers outlive every completion still held (the state's destructor also waits
// for its stream).
struct ckl_completion {
  std::shared_ptr<InvocationState> state;
  cudaEvent_t event = nullptr;
  ~ckl_completion() {
    if (event) {
      cudaSetDevice(state->device->ordinal);
      cudaEventDestroy(event);
    }
  }
};
struct ckl_graph_plan {
  ckl::planning::ProgramGraph graph;
  std::vector<uint32_t> resourceTemporary;
};

extern "C" {

const char *ckl_last_error(void) { return lastError.c_str(); }

int ckl_device_count(int *count) {
  return guarded([&] {
    if (!count)
      throw std::invalid_argument("null output");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    *count = n;
  });
}

int ckl_cuda_available(void) {
  int n = 0;
  return ckl_device_count(&n) == CKL_OK && n > 0 ? 1 : 0;
}

int ckl_device_create(int ordinal, ckl_device **out) {
  return guarded([&] {
    if (!out)
      throw std::invalid_argument("null output");
    int n = 0;
    check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    if (ordinal < 0 || ordinal >= n)
      throw std::invalid_argument("CUDA device ordinal out of range");
    auto d = std::make_shared<Device>();
    d->ordinal = ordinal;
    d->id = nextDeviceId++;
    d->current();
    check(cudaFree(nullptr), "cudaFree(context init)");
    cudaDeviceProp prop{};
    check(cudaGetDeviceProperties(&prop, ordinal), "cudaGetDeviceProperties");
    d->name = prop.name;
    *out = new ckl_device{d};
  });
}

void ckl_device_release(ckl_device *device) { delete device; }

int ckl_device_name(const ckl_device *device, char *name, size_t capacity) {
  return guarded([&] {
    if (!device || !name || !capacity)
      throw std::invalid_argument("invalid device name query");
    std::snprintf(name, capacity, "%s", device->device->name.c_str());
  });
}

int ckl_device_ordinal(const ckl_device *device) { return device ? device->device->ordinal : -1; }

int ckl_buffer_allocate(ckl_device *device, uint64_t bytes, ckl_buffer **out) {
  return guarded([&] {
    if (!device || !out)
      throw std::invalid_argument("buffer allocation requires a device");
    if (!bytes)
      throw std::invalid_argument("allocation size must be nonzero");
    device->device->current();
    auto a = std::make_shared<Allocation>();
    a->device = device->device;
    void *p = nullptr;
    check(cudaMalloc(&p, bytes), "cudaMalloc");
    a->pointer = reinterpret_cast<uint64_t>(p);
    a->bytes = bytes;
    *out = new ckl_buffer{a, 0, bytes};
  });
}

int ckl_buffer_import(ckl_device *device, uint64_t address, uint64_t bytes, ckl_buffer **out) {
  return guarded([&] {
    if (!device || !out || !address || !bytes)
      throw std::invalid_argument("imported buffer requires an address and size");
    auto a = std::make_shared<Allocation>();
    a->device = device->device;
    a->pointer = address;
    a->bytes = bytes;
    a->owned = false;
    *out = new ckl_buffer{a, 0, bytes};
  });
}

int ckl_buffer_slice(const ckl_buffer *buffer, uint64_t offset, uint64_t bytes, ckl_buffer **out) {
  return guarded([&] {
    if (!buffer || !out || !bytes || offset > buffer->bytes || bytes > buffer->bytes - offset)
      throw std::out_of_range("buffer slice exceeds its parent view");
    *out = new ckl_buffer{buffer->allocation, buffer->offset + offset, bytes};
  });
}

void ckl_buffer_release(ckl_buffer *buffer) { delete buffer; }
uint64_t ckl_buffer_address(const ckl_buffer *buffer) { return buffer ? buffer->address() : 0; }
uint64_t ckl_buffer_size(const ckl_buffer *buffer) { return buffer ? buffer->bytes : 0; }

int ckl_buffer_copy_from_host(const ckl_buffer *buffer, const void *source, uint64_t bytes) {
  return guarded([&] {
    if (!buffer || !source || bytes > buffer->bytes)
      throw std::out_of_range("host-to-device copy exceeds the buffer");
    buffer->allocation->device->current();
    buffer->allocation->device->settle();
    check(cudaMemcpy(reinterpret_cast<void *>(buffer->address()), source, bytes,
                     cudaMemcpyHostToDevice),
          "cudaMemcpy(host-to-device)");
    // Pageable copies may return after staging; execution streams are non-blocking, so wait
    // for the transfer itself before any of them can read the destination.
    check(cudaStreamSynchronize(cudaStreamLegacy), "cudaStreamSynchronize(host-to-device)");
  });
}

int ckl_buffer_copy_to_host(const ckl_buffer *buffer, void *destination, uint64_t bytes) {
  return guarded([&] {
    if (!buffer || !destination || bytes > buffer->bytes)
      throw std::out_of_range("device-to-host copy exceeds the buffer");
    buffer->allocation->device->current();
    buffer->allocation->device->settle();
    check(cudaMemcpy(destination, reinterpret_cast<void *>(buffer->address()), bytes,
                     cudaMemcpyDeviceToHost),
          "cudaMemcpy(device-to-host)");
  });
}

int ckl_buffer_fill_zero(const ckl_buffer *buffer) {
  return guarded([&] {
    if (!buffer)
      throw std::invalid_argument("cannot clear an empty buffer");
    buffer->allocation->device->current();
    check(cudaMemset(reinterpret_cast<void *>(buffer->address()), 0, buffer->bytes), "cudaMemset");
    check(cudaStreamSynchronize(cudaStreamLegacy), "cudaStreamSynchronize(clear)");
  });
}

int ckl_host_alloc(uint64_t bytes, void **out) {
  return guarded([&] {
    if (!out || !bytes)
      throw std::invalid_argument("pinned allocation requires a size");
    check(cudaMallocHost(out, bytes), "cudaMallocHost");
  });
}

void ckl_host_free(void *pointer) {
  if (pointer)
    cudaFreeHost(pointer);
}

int ckl_program_create(ckl_entry_fn entry, uint32_t count, const uint64_t *buffer_bytes,
                       const char *const *scalar_types, ckl_program *fallback, ckl_program **out) {
  return guarded([&] {
    if (!entry || !out || (count && (!buffer_bytes || !scalar_types)))
      throw std::invalid_argument("invalid host entry or argument metadata");
    auto s = std::make_shared<ProgramState>();
    s->entry = entry;
    for (uint32_t i = 0; i < count; ++i) {
      s->bufferBytes.push_back(buffer_bytes[i]);
      s->scalarTypes.emplace_back(scalar_types[i] ? scalar_types[i] : "");
    }
    s->fallback = fallback ? fallback->state : nullptr;
    *out = new ckl_program{s};
  });
}

int ckl_program_create_from_plan(const char *plan_text, ckl_program *fallback, ckl_program **out) {
  return guarded([&] {
    if (!out)
      throw std::invalid_argument("null output");
    auto s = std::make_shared<ProgramState>();
    s->plan = parsePlan(plan_text);
    s->entry = &planEntry;
    s->bufferBytes = s->plan->bufferBytes;
    s->scalarTypes = s->plan->scalarTypes;
    s->fallback = fallback ? fallback->state : nullptr;
    *out = new ckl_program{s};
  });
}

void ckl_program_release(ckl_program *program) { delete program; }

int ckl_bind(ckl_program *program, ckl_device *device, uint32_t count, const ckl_argument *args,
             ckl_invocation **out) {
  return guarded([&] {
    if (!program || !device || !out)
      throw std::invalid_argument("program binding requires a program and a device");
    auto p = program->state;
    if (count != p->bufferBytes.size() || (count && !args))
      throw std::invalid_argument("incorrect program argument count");
    std::vector<uint64_t> addresses(count), scalars(count);
    std::vector<void *> packed(count);
    std::vector<std::shared_ptr<Allocation>> keep;
    for (uint32_t i = 0; i < count; ++i) {
      if (p->bufferBytes[i]) {
        const ckl_buffer *b = args[i].kind == CKL_ARG_BUFFER ? args[i].buffer : nullptr;
        if (args[i].kind != CKL_ARG_BUFFER)
          throw std::invalid_argument("argument type does not match compiled signature");
        if (!b || b->allocation->device != device->device || b->bytes < p->bufferBytes[i])
          throw std::invalid_argument("buffer device or size does not match compiled signature");
        addresses[i] = b->address();
        packed[i] = &addresses[i];
        keep.push_back(b->allocation);
      } else {
        requireScalarType(p->scalarTypes[i], args[i].kind);
        scalars[i] = args[i].bits;
        packed[i] = &scalars[i];
      }
    }
    // Fused plans assume distinct buffers; overlapping bindings (including shifted views)
    // take the original kernel boundaries (NvidiaProgram.cpp:194-205).  A plan whose kernels
    // access caller buffers in wider units (the fused decoder: 16 bytes) states it, and a
    // buffer that does not start on such a boundary takes the original boundaries too.
    if (p->fallback) {
      bool overlap = false;
      const uint64_t alignment = p->plan ? p->plan->alignment : 1;
      for (uint32_t i = 0; i < count; ++i)
        overlap |= p->bufferBytes[i] != 0 && addresses[i] % alignment != 0;
      for (uint32_t i = 0; i < count; ++i)
        for (uint32_t j = i + 1; j < count; ++j) {
          if (!p->bufferBytes[i] || !p->bufferBytes[j])
            continue;
          overlap |= addresses[i] <= addresses[j] ? addresses[j] - addresses[i] < p->bufferBytes[i]
                                                  : addresses[i] - addresses[j] < p->bufferBytes[j];
        }
      if (overlap)
        p = p->fallback;
    }
    auto state = std::make_shared<InvocationState>();
    state->program = p;
    state->device = device->device;
    state->buffers = std::move(keep);
    state->device->current();
    check(cudaStreamCreateWithFlags(&state->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    void *frame = state.get();
    void **values = packed.data();
    void *entryArguments[] = {&frame, &values};
    p->entry(entryArguments);
    if (!state->error.empty())
      throw std::runtime_error(state->error);
    for (const KernelLaunch &k : state->plan.nodes)
      state->boundedWaits |= k.function.entry != nullptr && k.function.entry->boundedWaits;
    *out = new ckl_invocation{state};
  });
}

void ckl_invocation_release(ckl_invocation *invocation) { delete invocation; }

int ckl_run(ckl_invocation *invocation, int mode, uint64_t batch) {
  return guarded([&] {
    if (!invocation)
      throw std::invalid_argument("null invocation");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    validateExecution(f, mode, batch);
    f.device->current();
    submit(f, mode, batch);
    check(cudaStreamSynchronize(f.stream), "cudaStreamSynchronize");
    checkLibraryFaults(f);
  });
}

int ckl_launch(ckl_invocation *invocation, int mode, uint64_t batch) {
  return guarded([&] {
    if (!invocation)
      throw std::invalid_argument("null invocation");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    validateExecution(f, mode, batch);
    f.device->current();
    f.device->asyncPending = true;
    submit(f, mode, batch);
  });
}

int ckl_synchronize(ckl_invocation *invocation) {
  return guarded([&] {
    if (!invocation)
      throw std::invalid_argument("null invocation");
    auto &f = *invocation->state;
    f.device->current();
    check(cudaStreamSynchronize(f.stream), "cudaStreamSynchronize");
    checkLibraryFaults(f);
  });
}

int ckl_copy_in_async(ckl_invocation *invocation, const ckl_buffer *buffer, const void *source,
                      uint64_t bytes) {
  return guarded([&] {
    if (!invocation || !buffer || !source || bytes > buffer->bytes)
      throw std::out_of_range("asynchronous host-to-device copy exceeds the buffer");
    auto &f = *invocation->state;
    f.device->current();
    f.device->asyncPending = true;
    check(cudaMemcpyAsync(reinterpret_cast<void *>(buffer->address()), source, bytes,
                          cudaMemcpyHostToDevice, f.stream),
          "cudaMemcpyAsync(host-to-device)");
  });
}

int ckl_copy_out_async(ckl_invocation *invocation, const ckl_buffer *buffer, void *destination,
                       uint64_t bytes) {
  return guarded([&] {
    if (!invocation || !buffer || !destination || bytes > buffer->bytes)
      throw std::out_of_range("asynchronous device-to-host copy exceeds the buffer");
    auto &f = *invocation->state;
    f.device->current();
    f.device->asyncPending = true;
    check(cudaMemcpyAsync(destination, reinterpret_cast<void *>(buffer->address()), bytes,
                          cudaMemcpyDeviceToHost, f.stream),
          "cudaMemcpyAsync(device-to-host)");
  });
}

int ckl_record(ckl_invocation *invocation, ckl_completion **out) {
  return guarded([&] {
    if (!invocation || !out)
      throw std::invalid_argument("null invocation or completion output");
    *out = nullptr;
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    f.device->current();
    auto completion = std::make_unique<ckl_completion>();
    completion->state = invocation->state;
    check(cudaEventCreateWithFlags(&completion->event, cudaEventDisableTiming),
          "cudaEventCreateWithFlags");
    check(cudaEventRecord(completion->event, f.stream), "cudaEventRecord");
    *out = completion.release();
  });
}

int ckl_wait_for(ckl_invocation *invocation, const ckl_completion *completion) {
  return guarded([&] {
    if (!invocation || !completion)
      throw std::invalid_argument("null invocation or completion");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    f.device->current();
    f.device->asyncPending = true;
    check(cudaStreamWaitEvent(f.stream, completion->event, 0), "cudaStreamWaitEvent");
  });
}

int ckl_completion_query(const ckl_completion *completion, int *done) {
  return guarded([&] {
    if (!completion || !done)
      throw std::invalid_argument("null completion or output");
    completion->state->device->current();
    const cudaError_t status = cudaEventQuery(completion->event);
    if (status == cudaErrorNotReady) {
      cudaGetLastError();
      *done = 0;
      return;
    }
    check(status, "cudaEventQuery");
    *done = 1;
    checkLibraryFaults(*completion->state);
  });
}

int ckl_completion_wait(const ckl_completion *completion, uint64_t timeout_us, int *done) {
  return guarded([&] {
    if (!completion || !done)
      throw std::invalid_argument("null completion or output");
    completion->state->device->current();
    *done = 0;
    if (timeout_us == UINT64_MAX) {
      check(cudaEventSynchronize(completion->event), "cudaEventSynchronize");
      *done = 1;
      checkLibraryFaults(*completion->state);
      return;
    }
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(timeout_us);
    for (;;) {
      const cudaError_t status = cudaEventQuery(completion->event);
      if (status == cudaSuccess) {
        *done = 1;
        checkLibraryFaults(*completion->state);
        return;
      }
      if (status != cudaErrorNotReady)
        check(status, "cudaEventQuery");
      cudaGetLastError();
      if (std::chrono::steady_clock::now() >= deadline)
        return;
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  });
}

void ckl_completion_release(ckl_completion *completion) { delete completion; }

int ckl_benchmark(ckl_invocation *invocation, int mode, uint64_t iterations, uint64_t batch,
                  double out[3]) {
  return guarded([&] {
    if (!invocation || !out)
      throw std::invalid_argument("null invocation or output");
    if (!iterations)
      throw std::invalid_argument("benchmark iterations must be positive");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    validateExecution(f, mode, batch);
    f.device->current();
    using Clock = std::chrono::steady_clock;
    check(cudaStreamSynchronize(f.stream), "cudaStreamSynchronize");
    auto setup = Clock::now();
    if (mode)
      executionGraph(f, mode, batch);
    out[2] = std::chrono::duration<double, std::milli>(Clock::now() - setup).count();
    cudaEvent_t start = nullptr, stop = nullptr;
    check(cudaEventCreate(&start), "cudaEventCreate");
    std::unique_ptr<void, void (*)(void *)> startGuard(start, [](void *e) {
      cudaEventDestroy(static_cast<cudaEvent_t>(e));
    });
    check(cudaEventCreate(&stop), "cudaEventCreate");
    std::unique_ptr<void, void (*)(void *)> stopGuard(stop, [](void *e) {
      cudaEventDestroy(static_cast<cudaEvent_t>(e));
    });
    check(cudaEventRecord(start, f.stream), "cudaEventRecord");
    auto wall = Clock::now();
    for (uint64_t i = 0; i < iterations; ++i)
      submit(f, mode, batch);
    check(cudaEventRecord(stop, f.stream), "cudaEventRecord");
    check(cudaEventSynchronize(stop), "cudaEventSynchronize");
    auto wallStop = Clock::now();
    float elapsed = 0;
    check(cudaEventElapsedTime(&elapsed, start, stop), "cudaEventElapsedTime");
    checkLibraryFaults(f);
    out[0] = elapsed * 1000.0 / double(iterations) / double(batch);
    out[1] = std::chrono::duration<double, std::micro>(wallStop - wall).count() /
             double(iterations) / double(batch);
  });
}

int ckl_time_launches(ckl_invocation *invocation, int mode, uint64_t batch, uint64_t steps,
                      double *out_ms) {
  return guarded([&] {
    if (!invocation || !out_ms || !steps)
      throw std::invalid_argument("invalid timing request");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    validateExecution(f, mode, batch);
    f.device->current();
    if (mode)
      executionGraph(f, mode, batch);
    cudaEvent_t start = nullptr, stop = nullptr;
    check(cudaEventCreate(&start), "cudaEventCreate");
    check(cudaEventCreate(&stop), "cudaEventCreate");
    cudaError_t status = cudaEventRecord(start, f.stream);
    for (uint64_t i = 0; i < steps && status == cudaSuccess; ++i) {
      try {
        submit(f, mode, batch);
      } catch (...) {
        cudaEventDestroy(start);
        cudaEventDestroy(stop);
        throw;
      }
    }
    if (status == cudaSuccess)
      status = cudaEventRecord(stop, f.stream);
    if (status == cudaSuccess)
      status = cudaEventSynchronize(stop);
    float ms = 0;
    if (status == cudaSuccess)
      status = cudaEventElapsedTime(&ms, start, stop);
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    check(status, "event timing");
    checkLibraryFaults(f);
    *out_ms = ms;
  });
}

int ckl_profile_nodes(ckl_invocation *invocation, uint64_t iterations, double *out_ms,
                      uint64_t capacity) {
  return guarded([&] {
    if (!invocation || !out_ms || !iterations)
      throw std::invalid_argument("invalid profiling request");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    const std::size_t n = f.plan.nodes.size();
    if (capacity < n)
      throw std::out_of_range("profile output holds fewer entries than the plan has nodes");
    f.device->current();
    std::vector<cudaEvent_t> events(n + 1, nullptr);
    auto destroy = [&] {
      for (cudaEvent_t e : events)
        if (e)
          cudaEventDestroy(e);
    };
    try {
      for (auto &e : events)
        check(cudaEventCreate(&e), "cudaEventCreate");
      for (std::size_t i = 0; i < n; ++i)
        out_ms[i] = 0;
      for (uint64_t it = 0; it < iterations; ++it) {
        for (std::size_t i = 0; i < n; ++i) {
          check(cudaEventRecord(events[i], f.stream), "cudaEventRecord");
          launchOne(f.plan.nodes[i], f.stream);
        }
        check(cudaEventRecord(events[n], f.stream), "cudaEventRecord");
        check(cudaEventSynchronize(events[n]), "cudaEventSynchronize");
        for (std::size_t i = 0; i < n; ++i) {
          float ms = 0;
          check(cudaEventElapsedTime(&ms, events[i], events[i + 1]), "cudaEventElapsedTime");
          out_ms[i] += ms;
        }
      }
    } catch (...) {
      destroy();
      throw;
    }
    destroy();
    checkLibraryFaults(f);
  });
}

int ckl_node_argument_sizes(const ckl_invocation *invocation, uint64_t node, uint64_t *sizes,
                            uint32_t capacity, uint32_t *count) {
  return guarded([&] {
    if (!invocation || !count || (capacity && !sizes))
      throw std::invalid_argument("invalid node argument query");
    const auto &nodes = invocation->state->plan.nodes;
    if (node >= nodes.size())
      throw std::out_of_range("node index out of range");
    const KernelLaunch &k = nodes[node];
    const std::size_t slots =
        k.arguments.size() - (k.function.entry && k.function.entry->prepare ? 1 : 0);
    *count = uint32_t(slots);
    for (std::size_t i = 0; i < slots && i < capacity; ++i)
      sizes[i] = k.arguments[i].size();
  });
}

int ckl_update_kernel(ckl_invocation *invocation, int mode, uint64_t batch, uint64_t node,
                      uint32_t count, const void *const *arguments, const uint64_t *argument_bytes,
                      const uint32_t *grid, const uint32_t *block, int64_t shared) {
  return guarded([&] {
    if (!invocation)
      throw std::invalid_argument("null invocation");
    auto &f = *invocation->state;
    std::lock_guard<std::mutex> lock(f.runMutex);
    validateExecution(f, mode, batch);
    if (mode == 2)
      throw std::invalid_argument("captured graph node indices cannot be updated");
    if (mode != 1)
      throw std::invalid_argument("only an explicit graph (mode 1) has updatable kernel nodes");
    f.device->current();
    GraphExec &g = executionGraph(f, mode, batch);
    if (node >= g.nodes.size() || node >= g.launches.size())
      throw std::out_of_range("graph kernel update references an unknown node");
    KernelLaunch updated = g.launches[node];
    const ckl::library::Kernel *entry = updated.function.entry;
    const std::size_t slots = updated.arguments.size() - (entry && entry->prepare ? 1 : 0);
    if (count != slots || (count && (!arguments || !argument_bytes)))
      throw std::invalid_argument("graph kernel update: argument count does not match the node");
    for (uint32_t i = 0; i < count; ++i) {
      if (!arguments[i])
        continue; // keep this slot
      if (argument_bytes[i] != updated.arguments[i].size())
        throw std::invalid_argument("graph kernel update: argument " + std::to_string(i) +
                                    " has " + std::to_string(argument_bytes[i]) +
                                    " bytes, the node's slot " +
                                    std::to_string(updated.arguments[i].size()));
      std::memcpy(updated.arguments[i].data(), arguments[i], argument_bytes[i]);
    }
    if (grid)
      updated.grid = dim3(grid[0], grid[1], grid[2]);
    if (block)
      updated.block = dim3(block[0], block[1], block[2]);
    if (shared >= 0)
      updated.shared = unsigned(shared);
    const dim3 &gd = updated.grid, &bd = updated.block;
    if (!gd.x || !gd.y || !gd.z || !bd.x || !bd.y || !bd.z ||
        uint64_t(bd.x) * bd.y * bd.z > 1024 || gd.y > 65535 || gd.z > 65535 || gd.x >= (1u << 31))
      throw std::invalid_argument("graph kernel update: launch exceeds CUDA grid or block limits");
    if (updated.shared > g.launches[node].shared)
      throw std::invalid_argument("graph kernel update: more dynamic shared memory than the node "
                                  "was built with");
    if (entry && entry->select) {
      const void *spec = entry->specBytes ? updated.arguments[slots - 1].data() : nullptr;
      if (entry->select(spec) != updated.function.address)
        throw std::invalid_argument(std::string("graph kernel update: the new specialization of ") +
                                    entry->name + " needs another compiled configuration; bind "
                                    "again instead");
    }
    if (entry && entry->prepare) {
      // The extra parameter (for example a TMA tensor map of a weight buffer) follows the new
      // arguments.
      const void *spec = entry->specBytes ? updated.arguments[slots - 1].data() : nullptr;
      std::vector<const void *> pointers;
      for (std::size_t i = 0; i < slots; ++i)
        pointers.push_back(updated.arguments[i].data());
      if (!entry->prepare(spec, pointers.data(), pointers.size(), updated.arguments.back().data()))
        throw std::invalid_argument(std::string("graph kernel update: arguments not supported by ") +
                                    entry->name);
    }
    auto pointers = updated.pointers();
    cudaKernelNodeParams p{};
    p.func = const_cast<void *>(updated.function.address);
    p.gridDim = updated.grid;
    p.blockDim = updated.block;
    p.sharedMemBytes = updated.shared;
    p.kernelParams = pointers.data();
    check(cudaGraphExecKernelNodeSetParams(g.exec, g.nodes[node], &p),
          "cudaGraphExecKernelNodeSetParams");
    g.launches[node] = std::move(updated);
  });
}

int ckl_node_count(const ckl_invocation *invocation, uint64_t *out) {
  return guarded([&] {
    if (!invocation || !out)
      throw std::invalid_argument("null invocation");
    *out = invocation->state->plan.nodes.size();
  });
}

int ckl_node_name(const ckl_invocation *invocation, uint64_t node, char *name, size_t capacity) {
  return guarded([&] {
    if (!invocation || !name || !capacity)
      throw std::invalid_argument("invalid node query");
    const auto &nodes = invocation->state->plan.nodes;
    if (node >= nodes.size())
      throw std::out_of_range("node index out of range");
    std::snprintf(name, capacity, "%s", nodes[node].function.name.c_str());
  });
}

int ckl_profiler_start(void) {
  return guarded([] { check(cudaProfilerStart(), "cudaProfilerStart"); });
}
int ckl_profiler_stop(void) {
  return guarded([] { check(cudaProfilerStop(), "cudaProfilerStop"); });
}

// ---- callbacks -------------------------------------------------------------------------
void ckl_begin(void *frame, const void *binary, uint64_t bytes) {
  callback(frame, [&](InvocationState &f) {
    if (!binary || !bytes)
      throw std::invalid_argument("cannot load an empty device binary");
    std::lock_guard<std::mutex> lock(f.program->moduleMutex);
    auto &module = f.program->modules[f.device->id];
    if (!module) {
      auto m = std::make_shared<Module>();
      m->device = f.device;
      const auto *bytesIn = static_cast<const unsigned char *>(binary);
      std::string marker(kLibraryMarker);
      if (bytes == marker.size() && std::memcmp(binary, marker.data(), bytes) == 0) {
        m->library = true;
      } else if (bytes >= 4 && bytesIn[0] == 0x7f && bytesIn[1] == 'E' && bytesIn[2] == 'L' &&
                 bytesIn[3] == 'F') {
        m->library = false;
        f.device->current();
        check(cudaLibraryLoadData(&m->handle, binary, nullptr, nullptr, 0, nullptr, nullptr, 0),
              "cudaLibraryLoadData");
      } else {
        throw std::invalid_argument("device binary is neither a CUBIN nor the kernel library");
      }
      module = m;
    }
    f.module = module;
  });
}

void ckl_heap(void *frame, uint64_t id, uint64_t bytes) {
  callback(frame, [&](InvocationState &f) {
    if (!bytes)
      throw std::invalid_argument("heap size must be nonzero");
    if (f.heaps.size() <= id)
      f.heaps.resize(id + 1);
    auto a = std::make_shared<Allocation>();
    a->device = f.device;
    void *p = nullptr;
    f.device->current();
    check(cudaMalloc(&p, bytes), "cudaMalloc(heap)");
    a->pointer = reinterpret_cast<uint64_t>(p);
    a->bytes = bytes;
    // Heaps start zero-filled: persistent planner slots (completion counters) rely on it.
    check(cudaMemset(p, 0, bytes), "cudaMemset(heap)");
    check(cudaDeviceSynchronize(), "cudaDeviceSynchronize(heap)");
    f.heaps[id] = a;
  });
}

void ckl_resource(void *frame, uint64_t id, uint64_t heap, uint64_t offset, void *external) {
  callback(frame, [&](InvocationState &f) {
    if (f.resources.size() <= id)
      f.resources.resize(id + 1);
    if (external) {
      f.resources[id] = *static_cast<uint64_t *>(external);
    } else {
      const auto &h = f.heaps.at(heap);
      if (!h || offset > h->bytes)
        throw std::out_of_range("temporary resource lies outside its heap");
      f.resources[id] = h->pointer + offset;
    }
  });
}

void ckl_kernel(void *frame, const char *name, uint64_t gx, uint64_t gy, uint64_t gz, uint64_t bx,
                uint64_t by, uint64_t bz, uint64_t shared) {
  callback(frame, [&](InvocationState &f) {
    if (!f.module)
      throw std::invalid_argument("ckl_kernel before ckl_begin");
    if (!name)
      throw std::invalid_argument("kernel name is null");
    if (!gx || !gy || !gz || !bx || !by || !bz)
      throw std::invalid_argument("kernel plan node requires positive launch dimensions");
    if (bx * by * bz > 1024 || gx >= (1ull << 31) || gy > 65535 || gz > 65535)
      throw std::invalid_argument("kernel launch exceeds CUDA grid or block limits");
    Function fn;
    fn.module = f.module;
    fn.name = name;
    // Library kernels resolve by name in every plan; a plan with a CUBIN (generated kernels
    // or a hand-written module) resolves its other names in that module.
    const ckl::library::Kernel *entry = ckl::library::find(name);
    if (entry || f.module->library) {
      fn.entry = entry;
      if (!fn.entry)
        throw std::invalid_argument(std::string("unknown library kernel: ") + name);
      fn.address = fn.entry->function;
      // Entries that pick a configuration at commit raise the limit for the one they pick.
      if (shared > 48 * 1024 && !fn.entry->select) {
        f.device->current();
        check(cudaFuncSetAttribute(fn.address, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(shared)),
              "cudaFuncSetAttribute");
      }
    } else {
      cudaKernel_t kernel = nullptr;
      f.device->current();
      check(cudaLibraryGetKernel(&kernel, f.module->handle, name), "cudaLibraryGetKernel");
      fn.address = reinterpret_cast<const void *>(kernel);
      if (shared > 48 * 1024)
        check(cudaKernelSetAttributeForDevice(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(shared), f.device->ordinal),
              "cudaKernelSetAttributeForDevice");
    }
    f.pending = KernelLaunch{};
    f.pending.function = fn;
    f.pending.grid = dim3(unsigned(gx), unsigned(gy), unsigned(gz));
    f.pending.block = dim3(unsigned(bx), unsigned(by), unsigned(bz));
    f.pending.shared = unsigned(shared);
    f.pendingDeps.clear();
  });
}

void ckl_argument_resource(void *frame, uint64_t id, uint64_t offset) {
  callback(frame, [&](InvocationState &f) {
    uint64_t address = f.resources.at(id) + offset;
    std::vector<unsigned char> bytes(sizeof(address));
    std::memcpy(bytes.data(), &address, sizeof(address));
    f.pending.arguments.push_back(std::move(bytes));
  });
}

void ckl_argument_value(void *frame, const void *value, uint64_t bytes) {
  callback(frame, [&](InvocationState &f) {
    if (!value || !bytes)
      throw std::invalid_argument("physical kernel argument must not be empty");
    const auto *p = static_cast<const unsigned char *>(value);
    f.pending.arguments.emplace_back(p, p + bytes);
  });
}

void ckl_dependency(void *frame, uint64_t id) {
  callback(frame, [&](InvocationState &f) { f.pendingDeps.push_back(f.nodes.at(id)); });
}

void ckl_commit(void *frame, uint64_t id) {
  callback(frame, [&](InvocationState &f) {
    if (const ckl::library::Kernel *k = f.pending.function.entry) {
      std::string signature = k->signature;
      if (signature.size() != f.pending.arguments.size())
        throw std::invalid_argument(std::string("argument count does not match library kernel ") +
                                    k->name);
      for (std::size_t i = 0; i < signature.size(); ++i)
        if (ckl::library::slotBytes(signature[i], k->specBytes) != f.pending.arguments[i].size())
          throw std::invalid_argument(std::string("argument size does not match library kernel ") +
                                      k->name);
      if (k->select) {
        const void *spec = k->specBytes ? f.pending.arguments.back().data() : nullptr;
        const void *chosen = k->select(spec);
        if (!chosen)
          throw std::invalid_argument(std::string("no compiled configuration of ") + k->name +
                                      " for this specialization");
        f.pending.function.address = chosen;
        if (f.pending.shared > 48 * 1024) {
          f.device->current();
          check(cudaFuncSetAttribute(chosen, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(f.pending.shared)),
                "cudaFuncSetAttribute");
          // Tensor-core pair kernels may be compiled for 16-CTA clusters (a non-portable size
          // that each kernel must opt into); other kernels are unaffected by the permission.
          check(cudaFuncSetAttribute(chosen, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "cudaFuncSetAttribute");
        }
      }
      if (k->prepare) {
        const void *spec = k->specBytes ? f.pending.arguments.back().data() : nullptr;
        std::vector<const void *> slots;
        for (const auto &a : f.pending.arguments)
          slots.push_back(a.data());
        std::vector<unsigned char> extra(k->prepareBytes);
        f.device->current();
        if (!k->prepare(spec, slots.data(), slots.size(), extra.data()))
          throw std::invalid_argument(std::string("arguments not supported by library kernel ") +
                                      k->name);
        f.pending.arguments.push_back(std::move(extra));
      }
    }
    f.nodes[id] = f.plan.add(std::move(f.pending), std::move(f.pendingDeps));
    f.pending = KernelLaunch{};
    f.pendingDeps.clear();
  });
}

int ckl_runtime_symbols(ckl_runtime_symbol out[8]) {
  return guarded([&] {
    if (!out)
      throw std::invalid_argument("null output");
    out[0] = {"ckl_begin", reinterpret_cast<uintptr_t>(&ckl_begin)};
    out[1] = {"ckl_heap", reinterpret_cast<uintptr_t>(&ckl_heap)};
    out[2] = {"ckl_resource", reinterpret_cast<uintptr_t>(&ckl_resource)};
    out[3] = {"ckl_kernel", reinterpret_cast<uintptr_t>(&ckl_kernel)};
    out[4] = {"ckl_argument_resource", reinterpret_cast<uintptr_t>(&ckl_argument_resource)};
    out[5] = {"ckl_argument_value", reinterpret_cast<uintptr_t>(&ckl_argument_value)};
    out[6] = {"ckl_dependency", reinterpret_cast<uintptr_t>(&ckl_dependency)};
    out[7] = {"ckl_commit", reinterpret_cast<uintptr_t>(&ckl_commit)};
  });
}

// ---- kernel library --------------------------------------------------------------------
int ckl_library_geometry(const char *name, const void *spec, uint64_t spec_bytes,
                         uint32_t grid[3], uint32_t block[3], uint32_t *shared_bytes) {
  return guarded([&] {
    const ckl::library::Kernel *k = name ? ckl::library::find(name) : nullptr;
    if (!k)
      throw std::invalid_argument(std::string("unknown library kernel: ") + (name ? name : ""));
    if (spec_bytes != k->specBytes || (spec_bytes && !spec))
      throw std::invalid_argument(std::string("specialization size mismatch for ") + k->name);
    ckl::library::Geometry g;
    if (!k->geometry || !k->geometry(spec, spec_bytes, &g))
      throw std::invalid_argument(std::string("unsupported specialization for ") + k->name);
    for (int i = 0; i < 3; ++i) {
      grid[i] = g.grid[i];
      block[i] = g.block[i];
    }
    *shared_bytes = g.sharedBytes;
  });
}

int ckl_library_signature(const char *name, char *signature, size_t capacity) {
  return guarded([&] {
    const ckl::library::Kernel *k = name ? ckl::library::find(name) : nullptr;
    if (!k || !signature || !capacity)
      throw std::invalid_argument("unknown library kernel or null output");
    std::snprintf(signature, capacity, "%s", k->signature);
  });
}

uint32_t ckl_library_count(void) { return static_cast<uint32_t>(ckl::library::count()); }
const char *ckl_library_name(uint32_t index) {
  const ckl::library::Kernel *k = ckl::library::at(index);
  return k ? k->name : nullptr;
}

// ---- planning ----------------------------------------------------------------------------
int ckl_graph_plan_create(uint32_t node_count, const ckl_graph_node *nodes, uint32_t access_count,
                          const ckl_graph_access *accesses, uint32_t resource_count,
                          const ckl_graph_resource *resources, uint32_t flags,
                          ckl_graph_plan **out) {
  return guarded([&] {
    using namespace ckl::planning;
    if (!out || (node_count && !nodes) || (access_count && !accesses) ||
        (resource_count && !resources))
      throw std::invalid_argument("invalid graph description");
    std::vector<GraphNode> graph(node_count);
    for (uint32_t i = 0; i < node_count; ++i) {
      const ckl_graph_node &n = nodes[i];
      if (n.kind > CKL_NODE_FREE || uint64_t(n.first_access) + n.access_count > access_count)
        throw std::invalid_argument("graph node describes invalid accesses");
      graph[i].kind = n.kind == CKL_NODE_DISPATCH ? NodeKind::Dispatch
                      : n.kind == CKL_NODE_ALLOC  ? NodeKind::Alloc
                                                  : NodeKind::Free;
      graph[i].unknown = n.unknown != 0;
      for (uint32_t a = 0; a < n.access_count; ++a) {
        const ckl_graph_access &acc = accesses[n.first_access + a];
        Region region;
        if (acc.offset == -1)
          region.kind = Region::Whole;
        else if (acc.offset < 0)
          region.kind = Region::Unknown;
        else {
          region.kind = Region::Interval;
          region.offset = acc.offset;
          region.length = acc.length;
        }
        graph[i].accesses.push_back({acc.resource, acc.bits, region});
      }
    }
    std::vector<ProgramResource> res(resource_count);
    auto result = new ckl_graph_plan();
    for (uint32_t r = 0; r < resource_count; ++r) {
      res[r].temporary = resources[r].temporary != 0;
      res[r].persistent = resources[r].temporary == 2;
      res[r].device = resources[r].device;
      res[r].bytes = resources[r].bytes;
      res[r].alignment = resources[r].alignment;
      result->resourceTemporary.push_back(resources[r].temporary);
    }
    try {
      result->graph = inferGraph(graph, res, flags & CKL_PLAN_REUSE_STORAGE,
                                 flags & CKL_PLAN_EXTERNALS_DISJOINT);
    } catch (...) {
      delete result;
      throw;
    }
    *out = result;
  });
}

void ckl_graph_plan_release(ckl_graph_plan *plan) { delete plan; }

uint64_t ckl_graph_plan_edge_count(const ckl_graph_plan *plan) {
  return plan ? plan->graph.edges.size() : 0;
}

void ckl_graph_plan_edges(const ckl_graph_plan *plan, uint32_t *pairs) {
  if (!plan || !pairs)
    return;
  for (std::size_t i = 0; i < plan->graph.edges.size(); ++i) {
    pairs[2 * i] = uint32_t(plan->graph.edges[i].from);
    pairs[2 * i + 1] = uint32_t(plan->graph.edges[i].to);
  }
}

uint64_t ckl_graph_plan_dependency_count(const ckl_graph_plan *plan, uint32_t node) {
  if (!plan)
    return 0;
  auto found = plan->graph.dependencies.find(node);
  return found == plan->graph.dependencies.end() ? 0 : found->second.size();
}

void ckl_graph_plan_dependencies(const ckl_graph_plan *plan, uint32_t node, uint32_t *out) {
  if (!plan || !out)
    return;
  auto found = plan->graph.dependencies.find(node);
  if (found == plan->graph.dependencies.end())
    return;
  for (std::size_t i = 0; i < found->second.size(); ++i)
    out[i] = uint32_t(found->second[i]);
}

uint64_t ckl_graph_plan_resource_count(const ckl_graph_plan *plan) {
  return plan ? plan->graph.resourceOrder.size() : 0;
}

void ckl_graph_plan_resources(const ckl_graph_plan *plan, uint32_t *out) {
  if (!plan || !out)
    return;
  for (std::size_t i = 0; i < plan->graph.resourceOrder.size(); ++i)
    out[i] = uint32_t(plan->graph.resourceOrder[i]);
}

void ckl_graph_plan_memory(const ckl_graph_plan *plan, uint64_t *baseline, uint64_t *planned,
                           uint32_t *heaps) {
  if (!plan)
    return;
  if (baseline)
    *baseline = plan->graph.memory.baselineBytes;
  if (planned)
    *planned = plan->graph.memory.plannedBytes;
  if (heaps)
    *heaps = uint32_t(plan->graph.memory.heaps.size());
}

void ckl_graph_plan_heaps(const ckl_graph_plan *plan, uint64_t *bytes, uint64_t *alignment) {
  if (!plan)
    return;
  for (std::size_t i = 0; i < plan->graph.memory.heaps.size(); ++i) {
    if (bytes)
      bytes[i] = plan->graph.memory.heaps[i].bytes;
    if (alignment)
      alignment[i] = plan->graph.memory.heaps[i].alignment;
  }
}

int ckl_graph_plan_assignment(const ckl_graph_plan *plan, uint32_t resource, uint64_t *heap,
                              uint64_t *offset, uint64_t *slot) {
  return guarded([&] {
    if (!plan)
      throw std::invalid_argument("null plan");
    const auto &g = plan->graph;
    for (std::size_t i = 0; i < g.plannerToProgram.size(); ++i)
      if (g.plannerToProgram[i] == resource) {
        const ckl::planning::Assignment *a = g.memory.find(i);
        if (!a)
          break;
        if (heap)
          *heap = a->heap;
        if (offset)
          *offset = a->offset;
        if (slot)
          *slot = a->slot;
        return;
      }
    throw std::out_of_range("resource has no memory-plan assignment");
  });
}

int ckl_memory_plan(uint32_t node_count, uint32_t edge_count, const uint32_t *edges,
                    uint32_t resource_count, const uint64_t *bytes, const uint64_t *alignment,
                    const uint32_t *kinds, const uint32_t *users_offsets, const uint32_t *users,
                    int reuse_storage, uint64_t *baseline_bytes, uint64_t *planned_bytes,
                    uint64_t *slots, uint64_t *offsets) {
  return guarded([&] {
    using namespace ckl::planning;
    std::vector<GraphEdge> e;
    for (uint32_t i = 0; i < edge_count; ++i)
      e.push_back({edges[2 * i], edges[2 * i + 1]});
    std::vector<PlannerResource> r(resource_count);
    for (uint32_t i = 0; i < resource_count; ++i) {
      r[i].bytes = bytes[i];
      r[i].alignment = alignment[i];
      r[i].kind = kinds[i] == 0 ? ResourceKind::Temporary
                  : kinds[i] == 1 ? ResourceKind::Persistent
                                  : ResourceKind::External;
      for (uint32_t u = users_offsets[i]; u < users_offsets[i + 1]; ++u)
        r[i].users.push_back(users[u]);
    }
    MemoryPlan plan = MemoryPlanner(reuse_storage != 0).plan(node_count, e, r);
    *baseline_bytes = plan.baselineBytes;
    *planned_bytes = plan.plannedBytes;
    for (uint32_t i = 0; i < resource_count; ++i) {
      const Assignment *a = plan.find(i);
      slots[i] = a ? a->slot : UINT64_MAX;
      offsets[i] = a ? a->offset : UINT64_MAX;
    }
  });
}

int ckl_repeat_dependencies(uint32_t node_count, const uint32_t *offsets, const uint32_t *deps,
                            uint32_t iterations, uint32_t *out_offsets, uint32_t *out_deps,
                            uint64_t out_capacity) {
  return guarded([&] {
    std::vector<std::vector<std::size_t>> in(node_count);
    for (uint32_t i = 0; i < node_count; ++i)
      for (uint32_t k = offsets[i]; k < offsets[i + 1]; ++k)
        in[i].push_back(deps[k]);
    auto result = ckl::planning::repeatDependencies(in, iterations);
    uint64_t total = 0;
    out_offsets[0] = 0;
    for (std::size_t i = 0; i < result.size(); ++i) {
      for (std::size_t d : result[i]) {
        if (total >= out_capacity)
          throw std::out_of_range("repeat output capacity exceeded");
        out_deps[total++] = uint32_t(d);
      }
      out_offsets[i + 1] = uint32_t(total);
    }
  });
}

} // extern "C"
