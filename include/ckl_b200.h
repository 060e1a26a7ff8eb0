/* C ABI of the CKL B200 runtime (libckl_b200.so).
 *
 * Plain pointers, sizes and status codes; no C++ or framework types cross this boundary.
 * Every function that can fail returns a status (CKL_OK == 0) and records a message that
 * ckl_last_error() returns on the same thread.  Each declaration names the reference
 * interface it replaces (paths inside the reference checkout).
 */
#ifndef CKL_B200_H
#define CKL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status ------------------------------------------------------------------------ */
enum {
  CKL_OK = 0,
  CKL_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument -> Python ValueError */
  CKL_RUNTIME_ERROR = 2,    /* reference: DriverError / std::runtime_error -> RuntimeError */
  CKL_OUT_OF_RANGE = 3      /* reference: std::out_of_range */
};

/* Thread-local message of the last failing call on this thread.
 * Replaces: DriverError messages, lib/Runtime/NvidiaRuntime.cpp:13-29. */
const char *ckl_last_error(void);

/* 1 when a CUDA device is usable, else 0.  Replaces: nvidiaDeviceAvailable(),
 * lib/Runtime/NvidiaProgram.cpp:283-286 (and _ckl_native.cuda_available). */
int ckl_cuda_available(void);
int ckl_device_count(int *count);

/* ---- devices ------------------------------------------------------------------------ */
typedef struct ckl_device ckl_device;
/* Replaces: NvidiaProgramDevice() / NvidiaRuntime(int deviceOrdinal),
 * include/ckl/Runtime/NvidiaProgram.h:16-20, lib/Runtime/NvidiaRuntime.cpp:222-230.
 * Any ordinal is accepted (the reference is device-0 only). */
int ckl_device_create(int ordinal, ckl_device **out);
void ckl_device_release(ckl_device *device);
int ckl_device_name(const ckl_device *device, char *name, size_t capacity);
int ckl_device_ordinal(const ckl_device *device);

/* ---- buffers ------------------------------------------------------------------------ */
typedef struct ckl_buffer ckl_buffer;
/* Replaces: NvidiaRuntime::allocate, lib/Runtime/NvidiaRuntime.cpp:248-257. */
int ckl_buffer_allocate(ckl_device *device, uint64_t bytes, ckl_buffer **out);
/* Borrowed device memory, never freed by CKL.  Replaces: NvidiaRuntime::importBuffer,
 * lib/Runtime/NvidiaRuntime.cpp:259-268. */
int ckl_buffer_import(ckl_device *device, uint64_t address, uint64_t bytes, ckl_buffer **out);
/* Bounded view sharing ownership.  Replaces: NvidiaBuffer::slice, NvidiaRuntime.cpp:150-154. */
int ckl_buffer_slice(const ckl_buffer *buffer, uint64_t offset, uint64_t bytes, ckl_buffer **out);
void ckl_buffer_release(ckl_buffer *buffer);
uint64_t ckl_buffer_address(const ckl_buffer *buffer);
uint64_t ckl_buffer_size(const ckl_buffer *buffer);
/* Synchronous copies; host-to-device waits for device completion even from pageable memory.
 * Replaces: NvidiaBuffer::copyFromHost/copyToHost, NvidiaRuntime.cpp:124-140. */
int ckl_buffer_copy_from_host(const ckl_buffer *buffer, const void *source, uint64_t bytes);
int ckl_buffer_copy_to_host(const ckl_buffer *buffer, void *destination, uint64_t bytes);
/* Replaces: NvidiaBuffer::fillZero, NvidiaRuntime.cpp:142-148. */
int ckl_buffer_fill_zero(const ckl_buffer *buffer);
/* Page-locked host memory for asynchronous copies (no reference counterpart: the reference
 * copies synchronously from pageable memory). */
int ckl_host_alloc(uint64_t bytes, void **out);
void ckl_host_free(void *pointer);

/* ---- programs and invocations ---------------------------------------------------------- */
typedef struct ckl_program ckl_program;
typedef struct ckl_invocation ckl_invocation;

/* The packed host entry the reference JIT-compiles from ckl_exec (ExecToLLVM.cpp:25-120):
 * entry(packed) with packed[0] = &frame, packed[1] = &argument_pointer_array. */
typedef void (*ckl_entry_fn)(void **packed);

/* Program from an entry function and argument metadata: buffer byte sizes (0 for scalars)
 * and scalar type names ("i32", "i64", "f32", "f64"; "" for buffers).  `fallback` (may be
 * NULL) is used when two buffer arguments overlap.  Replaces: NvidiaProgram::NvidiaProgram,
 * lib/Runtime/NvidiaProgram.cpp:136-146. */
int ckl_program_create(ckl_entry_fn entry, uint32_t count, const uint64_t *buffer_bytes,
                       const char *const *scalar_types, ckl_program *fallback, ckl_program **out);
/* Program from a textual executable plan (heaps, resources, kernels, dependencies); its
 * built-in entry replays the plan through the eight callbacks below in the order the
 * reference's generated entry uses.  Replaces: the JIT-compiled ckl_entry of
 * python/ckl/_jit.py:126-154 + lib/Transforms/ExecToLLVM.cpp:25-120. */
int ckl_program_create_from_plan(const char *plan_text, ckl_program *fallback, ckl_program **out);
void ckl_program_release(ckl_program *program);

enum { CKL_ARG_BUFFER = 0, CKL_ARG_I32 = 1, CKL_ARG_I64 = 2, CKL_ARG_F32 = 3, CKL_ARG_F64 = 4 };
typedef struct {
  uint32_t kind;      /* CKL_ARG_* */
  uint32_t reserved;
  ckl_buffer *buffer; /* CKL_ARG_BUFFER */
  uint64_t bits;      /* scalar value bits, little endian, zero extended */
} ckl_argument;

/* Bind arguments: validates, allocates temporary heaps, builds the bound plan.
 * Replaces: NvidiaProgram::bind, lib/Runtime/NvidiaProgram.cpp:156-215. */
int ckl_bind(ckl_program *program, ckl_device *device, uint32_t count, const ckl_argument *args,
             ckl_invocation **out);
void ckl_invocation_release(ckl_invocation *invocation);

/* Modes: 0 ordinary launches, 1 inferred-dependency graph, 2 single-stream capture.
 * `batch` repeats the whole program inside one submission.  Synchronous.
 * Replaces: NvidiaInvocation::run, lib/Runtime/NvidiaProgram.cpp:217-223. */
int ckl_run(ckl_invocation *invocation, int mode, uint64_t batch);
/* out[0] stream us per program, out[1] wall us per program, out[2] graph setup ms.
 * Replaces: NvidiaInvocation::benchmark, lib/Runtime/NvidiaProgram.cpp:225-270. */
int ckl_benchmark(ckl_invocation *invocation, int mode, uint64_t iterations, uint64_t batch,
                  double out[3]);
/* Replaces: NvidiaInvocation::nodeCount, NvidiaProgram.cpp:155. */
int ckl_node_count(const ckl_invocation *invocation, uint64_t *out);
/* Kernel nodes of one program execution with their reduced predecessors, for inspection:
 * names[i] receives at most `capacity` bytes. */
int ckl_node_name(const ckl_invocation *invocation, uint64_t node, char *name, size_t capacity);
/* Byte sizes of plan node `node`'s argument slots, in order (*count receives the number of
 * slots; at most `capacity` sizes are written).  No reference counterpart: it tells a caller
 * of ckl_update_kernel what each slot holds (8 for a pointer or i64/f64, 4 for i32/f32, the
 * specialization struct's size for a library kernel's last slot). */
int ckl_node_argument_sizes(const ckl_invocation *invocation, uint64_t node, uint64_t *sizes,
                            uint32_t capacity, uint32_t *count);
/* Replaces kernel node `node`'s launch parameters in the invocation's instantiated explicit
 * graph for `batch` repetitions (built on first use), without re-instantiating it
 * (cudaGraphExecKernelNodeSetParams).  Graph node r * node_count + i is repetition r's plan
 * node i.  `arguments[i]` points at `argument_bytes[i]` new bytes for slot i (the slot's own
 * size), or is NULL to keep the slot; `count` must be the node's slot count.  `grid` and
 * `block` (three values each) replace the launch shape when non-NULL, `shared` (>= 0, at most
 * the node's original amount) the dynamic shared memory.  The kernel stays the same: a new
 * specialization that needs another compiled configuration is rejected.  Library kernels that
 * derive a bind-time parameter from their arguments (the tensor-core kernels' TMA weight maps)
 * derive it again.  The update applies to that graph only; ordinary launches and other
 * graphs keep the bound plan.  Mode 2 (a captured graph, whose node indices are not stable)
 * and mode 0 are rejected.  Replaces: NvidiaGraphExecutable::updateKernel,
 * lib/Runtime/NvidiaRuntime.cpp:466-496. */
int ckl_update_kernel(ckl_invocation *invocation, int mode, uint64_t batch, uint64_t node,
                      uint32_t count, const void *const *arguments, const uint64_t *argument_bytes,
                      const uint32_t *grid, const uint32_t *block, int64_t shared);

/* Asynchronous submission on the invocation's stream (no reference counterpart; the
 * reference's only mode is synchronous).  Pair with ckl_synchronize. */
int ckl_launch(ckl_invocation *invocation, int mode, uint64_t batch);
int ckl_synchronize(ckl_invocation *invocation);
int ckl_copy_in_async(ckl_invocation *invocation, const ckl_buffer *buffer, const void *source,
                      uint64_t bytes);
int ckl_copy_out_async(ckl_invocation *invocation, const ckl_buffer *buffer, void *destination,
                       uint64_t bytes);

/* Completions: the asynchronous invocation/completion interface the reference names as next
 * work (benchmarks/decoder/results/deep-dive/REPORT.md:155-159; its runs are synchronous,
 * lib/Runtime/NvidiaProgram.cpp:217-229).  ckl_record marks the current end of the
 * invocation's stream (after ckl_launch and asynchronous copies); the completion keeps the
 * invocation's stream, heaps and bound buffers alive until released.  ckl_wait_for makes an
 * invocation's later work wait on the device for another invocation's completion (also
 * across devices).  ckl_completion_wait polls up to timeout_us microseconds (UINT64_MAX:
 * blocks) and sets *done.  Synchronous buffer copies wait for a device's outstanding
 * asynchronous work before they touch its memory. */
typedef struct ckl_completion ckl_completion;
int ckl_record(ckl_invocation *invocation, ckl_completion **out);
int ckl_wait_for(ckl_invocation *invocation, const ckl_completion *completion);
int ckl_completion_query(const ckl_completion *completion, int *done);
int ckl_completion_wait(const ckl_completion *completion, uint64_t timeout_us, int *done);
void ckl_completion_release(ckl_completion *completion);
/* Device time of `steps` submissions of (mode, batch) bracketed by events on the invocation
 * stream; nothing else is enqueued in between.  out_ms receives the elapsed milliseconds. */
int ckl_time_launches(ckl_invocation *invocation, int mode, uint64_t batch, uint64_t steps,
                      double *out_ms);

/* Per-kernel device time: `iterations` ordinary executions of the bound plan with an event
 * pair around every node; out_ms[i] accumulates node i (capacity >= node count).  Each
 * iteration is a real execution of the program (state advances).  No reference counterpart
 * (the reference profiles with nsys, benchmarks/decoder/collect.py:14-96). */
int ckl_profile_nodes(ckl_invocation *invocation, uint64_t iterations, double *out_ms,
                      uint64_t capacity);

/* CUDA profiler range.  Replaces: nvidiaProfilerStart/Stop, NvidiaProgram.cpp:287-294. */
int ckl_profiler_start(void);
int ckl_profiler_stop(void);

/* ---- plan-building callbacks ----------------------------------------------------------- */
/* The eight callbacks the packed entry calls, with the reference's exact signatures and
 * error latch: the first failure is recorded, later callbacks become no-ops and binding
 * reports the error.  Replaces: lib/Runtime/NvidiaProgram.cpp:60-108 (exported as
 * nvidiaProgramRuntimeSymbols(), :272-281).  `binary` in ckl_begin is either a CUBIN for
 * sm_100a or the marker "ckl-b200:library", which selects the linked kernel library. */
void ckl_begin(void *frame, const void *binary, uint64_t bytes);
void ckl_heap(void *frame, uint64_t id, uint64_t bytes);
void ckl_resource(void *frame, uint64_t id, uint64_t heap, uint64_t offset, void *external);
void ckl_kernel(void *frame, const char *name, uint64_t gx, uint64_t gy, uint64_t gz,
                uint64_t bx, uint64_t by, uint64_t bz, uint64_t shared);
void ckl_argument_resource(void *frame, uint64_t id, uint64_t offset);
void ckl_argument_value(void *frame, const void *value, uint64_t bytes);
void ckl_dependency(void *frame, uint64_t id);
void ckl_commit(void *frame, uint64_t id);

typedef struct {
  const char *name;
  uintptr_t address;
} ckl_runtime_symbol;
/* Writes the eight callback symbols into out[0..7].  Replaces:
 * nvidiaProgramRuntimeSymbols(), NvidiaProgram.cpp:272-281. */
int ckl_runtime_symbols(ckl_runtime_symbol out[8]);

/* ---- kernel library --------------------------------------------------------------------- */
/* Launch geometry the library chooses for one of its kernels given its specialization
 * constants (no counterpart: the reference's geometry comes from each ckl.launch).
 * signature receives the kernel's parameter-slot code ('P' pointer, 'I' i32, 'L' i64,
 * 'F' f32, 'D' f64, 'S' specialization bytes). */
int ckl_library_geometry(const char *name, const void *spec, uint64_t spec_bytes,
                         uint32_t grid[3], uint32_t block[3], uint32_t *shared_bytes);
int ckl_library_signature(const char *name, char *signature, size_t capacity);
/* Fault word of the kernel library on the current device: bit 0 is set when a tensor-core
 * kernel gave up a bounded wait (it then skipped its work instead of hanging), bit 1 when it
 * found a misaligned operand.  `reset` clears the word after reading it.  While the word is
 * nonzero, every synchronizing call (ckl_run, ckl_synchronize, ckl_benchmark,
 * ckl_time_launches, ckl_profile_nodes, a completed ckl_completion_query/_wait) of an
 * invocation that contains such a kernel returns CKL_RUNTIME_ERROR.  No reference
 * counterpart (the reference's kernels never wait on the device). */
int ckl_library_faults(uint32_t *out, int reset);
/* Limit, in nanoseconds, of the tensor-core kernels' pipeline waits on device `device` for
 * launches made after the call (default 2000000000, two seconds).  The waits with which an
 * aborting CTA drains its own copies and MMAs keep a fixed two-second limit.  No reference
 * counterpart; used by tests to make a wait expire quickly. */
int ckl_set_wait_limit(int device, uint64_t nanoseconds);
/* Test hook (no reference counterpart): while `enable` is nonzero, every tensor-core kernel
 * CTA launched on `device` first waits on an mbarrier that nothing signals.  The wait expires
 * after the wait limit, sets fault bit 0 and takes the abort path, so the submission's
 * synchronizing call reports the fault and the context stays usable. */
int ckl_inject_unsignalled_wait(int device, int enable);
uint32_t ckl_library_count(void);
const char *ckl_library_name(uint32_t index);

/* Greedy LM head that allocates nothing (no counterpart in the reference).  For callers
 * that cannot allocate device memory where they run the head: logits = RMSNorm(x; gain,
 * eps) @ lm, tokens[b] = first-index argmax of logits[b], history[position * batch + b] =
 * tokens[b], position += 1, enqueued on `stream` (NULL: the default stream).  x: [batch,
 * hidden], gain: [hidden], lm: [hidden, vocab], logits: [batch, vocab], tokens: [batch],
 * history: [capacity, batch], position: [1], all device pointers.  Its scratch (argmax
 * partials and a completion counter) is a fixed 4 MiB array in the library's device memory:
 * batch * ceil(vocab / tile width) may not exceed 524288 partials (rejected with
 * CKL_INVALID_ARGUMENT).  All calls on a device share that array: calls that overlap on the
 * GPU race.  The first call on a device resolves the array's address (cudaGetSymbolAddress);
 * make it before any stream capture on that device.  The address is kept per device ordinal
 * for the life of the process: calls after a cudaDeviceReset, or under a context other than
 * the device's primary context, are not supported. */
int ckl_greedy_head_noalloc(const float *x, const float *gain, const float *lm, float eps,
                            int64_t batch, int64_t hidden, int64_t vocab, int64_t capacity,
                            float *logits, int32_t *tokens, int32_t *history, int32_t *position,
                            void *stream);

/* ---- generated kernels (no GPU needed) ---------------------------------------------------- */
/* Compiles CUDA C++ source (the frontend's translation of kernel bodies the library does not
 * implement) for sm_100a with NVRTC, loaded at run time: no multiply-add contraction, IEEE
 * division and square root, denormals kept.  On success *binary is a malloc'd CUBIN of *bytes
 * bytes (release with ckl_binary_free); a compile error is CKL_INVALID_ARGUMENT with NVRTC's
 * log in ckl_last_error().  Replaces: the NVVM lowering and gpu-module-to-binary serializer of
 * the reference's device pipeline, python/ckl/_jit.py:32-52. */
int ckl_cuda_compile(const char *source, const char *name, void **binary, uint64_t *bytes);
void ckl_binary_free(void *binary);

/* ---- planning (no GPU needed) ------------------------------------------------------------ */
/* Inference of the dependency graph, its transitive reduction onto dispatch nodes and the
 * temporary-storage plan of one traced program.  Replaces: buildGraph + attachMemoryPlan
 * (lib/Analysis/GraphAnalysis.cpp:143-600), getReducedDispatchDependencies
 * (lib/Analysis/GraphAlgorithms.cpp:10-46) and MemoryPlanner::plan
 * (lib/Core/MemoryPlanner.cpp:98-204). */
enum { CKL_NODE_DISPATCH = 0, CKL_NODE_ALLOC = 1, CKL_NODE_FREE = 2 };
enum { CKL_ACCESS_READ = 1, CKL_ACCESS_WRITE = 2, CKL_ACCESS_ALLOCATE = 4, CKL_ACCESS_FREE = 8 };
typedef struct {
  uint32_t kind;    /* CKL_NODE_* */
  uint32_t unknown; /* opaque effects: ordered against every other node */
  uint32_t first_access;
  uint32_t access_count;
} ckl_graph_node;
typedef struct {
  uint32_t resource;
  uint32_t bits;    /* CKL_ACCESS_* */
  int64_t offset;   /* byte interval start; -1 whole buffer, -2 unknown */
  int64_t length;
} ckl_graph_access;
typedef struct {
  uint32_t temporary; /* 0: caller buffer; 1: compiler temporary (fresh identity, reusable
                         storage); 2: persistent compiler storage (never shared; zeroed) */
  int32_t device;
  uint64_t bytes;
  uint64_t alignment;
} ckl_graph_resource;
enum { CKL_PLAN_REUSE_STORAGE = 1, CKL_PLAN_EXTERNALS_DISJOINT = 2 };
typedef struct ckl_graph_plan ckl_graph_plan;
int ckl_graph_plan_create(uint32_t node_count, const ckl_graph_node *nodes,
                          uint32_t access_count, const ckl_graph_access *accesses,
                          uint32_t resource_count, const ckl_graph_resource *resources,
                          uint32_t flags, ckl_graph_plan **out);
void ckl_graph_plan_release(ckl_graph_plan *plan);
uint64_t ckl_graph_plan_edge_count(const ckl_graph_plan *plan);
void ckl_graph_plan_edges(const ckl_graph_plan *plan, uint32_t *from_to_pairs);
uint64_t ckl_graph_plan_dependency_count(const ckl_graph_plan *plan, uint32_t node);
void ckl_graph_plan_dependencies(const ckl_graph_plan *plan, uint32_t node, uint32_t *out);
/* Resources in first-access order over dispatch nodes (the plan's resource numbering). */
uint64_t ckl_graph_plan_resource_count(const ckl_graph_plan *plan);
void ckl_graph_plan_resources(const ckl_graph_plan *plan, uint32_t *out);
void ckl_graph_plan_memory(const ckl_graph_plan *plan, uint64_t *baseline_bytes,
                           uint64_t *planned_bytes, uint32_t *heap_count);
void ckl_graph_plan_heaps(const ckl_graph_plan *plan, uint64_t *bytes, uint64_t *alignment);
/* 0 and heap/offset/slot of a planned temporary; CKL_OUT_OF_RANGE for caller buffers. */
int ckl_graph_plan_assignment(const ckl_graph_plan *plan, uint32_t resource, uint64_t *heap,
                              uint64_t *offset, uint64_t *slot);

/* Stand-alone memory planner over explicit lifetimes (tests; MemoryPlanner::plan).
 * kinds: 0 temporary, 1 persistent, 2 external.  users_offsets has resource_count+1 entries.
 * Outputs per resource: slot (UINT64_MAX for external), heap offset.  */
int ckl_memory_plan(uint32_t node_count, uint32_t edge_count, const uint32_t *edges,
                    uint32_t resource_count, const uint64_t *bytes, const uint64_t *alignment,
                    const uint32_t *kinds, const uint32_t *users_offsets, const uint32_t *users,
                    int reuse_storage, uint64_t *baseline_bytes, uint64_t *planned_bytes,
                    uint64_t *slots, uint64_t *offsets);
/* Predecessors of `batch` repetitions of a dependency list (ExecutionPlan::repeat,
 * lib/Core/ExecutionPlan.cpp:87-117); CSR in/out. */
int ckl_repeat_dependencies(uint32_t node_count, const uint32_t *offsets, const uint32_t *deps,
                            uint32_t iterations, uint32_t *out_offsets, uint32_t *out_deps,
                            uint64_t out_capacity);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* CKL_B200_H */
