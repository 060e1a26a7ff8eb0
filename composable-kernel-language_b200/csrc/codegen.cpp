// Device compilation of generated CKL kernels: CUDA C++ source -> sm_100a CUBIN with NVRTC.
//
// The reference serializes its kernel module with MLIR's gpu-lower-to-nvvm-pipeline and
// gpu-module-to-binary (python/ckl/_jit.py:32-52, chip and features from NVIDIATarget).  Here
// the frontend emits CUDA C++ for the kernels the library does not implement and this entry
// compiles them in process.  NVRTC is loaded at run time (dlopen), so the library still loads
// where no CUDA toolkit is installed; compilation then fails with a message.  Options: sm_100a,
// no multiply-add contraction, IEEE division and square root, denormals preserved (the
// reference's NVPTX defaults without fast-math flags).
#include "ckl_b200.h"
#include "errors.hpp"

#include <nvrtc.h>

#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

struct Nvrtc {
  void *handle = nullptr;
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) logSize = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubinSize = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  decltype(&nvrtcGetErrorString) error = nullptr;
  std::string failure;
};

template <typename T> void resolve(Nvrtc &n, T &slot, const char *name) {
  slot = reinterpret_cast<T>(dlsym(n.handle, name));
  if (!slot)
    n.failure = std::string("NVRTC lacks ") + name;
}

const Nvrtc &nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    std::vector<std::string> candidates;
    if (const char *configured = std::getenv("CKL_B200_NVRTC"))
      candidates.emplace_back(configured);
    candidates.emplace_back("libnvrtc.so.12");
    candidates.emplace_back("/usr/local/cuda/lib64/libnvrtc.so.12");
    candidates.emplace_back("libnvrtc.so");
    for (const auto &path : candidates)
      if ((n.handle = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL)))
        break;
    if (!n.handle) {
      n.failure = "NVRTC (libnvrtc.so.12) could not be loaded; set CKL_B200_NVRTC";
      return;
    }
    resolve(n, n.create, "nvrtcCreateProgram");
    resolve(n, n.compile, "nvrtcCompileProgram");
    resolve(n, n.logSize, "nvrtcGetProgramLogSize");
    resolve(n, n.log, "nvrtcGetProgramLog");
    resolve(n, n.cubinSize, "nvrtcGetCUBINSize");
    resolve(n, n.cubin, "nvrtcGetCUBIN");
    resolve(n, n.destroy, "nvrtcDestroyProgram");
    resolve(n, n.error, "nvrtcGetErrorString");
  });
  return n;
}

void require(const Nvrtc &n, nvrtcResult status, const char *operation) {
  if (status != NVRTC_SUCCESS)
    throw std::runtime_error(std::string(operation) + " failed: " + n.error(status));
}

} // namespace

int ckl_cuda_compile(const char *source, const char *name, void **binary, uint64_t *bytes) {
  try {
    if (!source || !binary || !bytes)
      throw std::invalid_argument("ckl_cuda_compile needs source, binary and bytes");
    *binary = nullptr;
    *bytes = 0;
    const Nvrtc &n = nvrtc();
    if (!n.failure.empty())
      throw std::runtime_error(n.failure);
    nvrtcProgram program = nullptr;
    require(n, n.create(&program, source, name ? name : "ckl_generated.cu", 0, nullptr, nullptr),
            "nvrtcCreateProgram");
    const char *options[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--prec-div=true",
                             "--prec-sqrt=true", "--ftz=false", "--std=c++17", "-lineinfo"};
    const nvrtcResult compiled =
        n.compile(program, int(sizeof(options) / sizeof(options[0])), options);
    if (compiled != NVRTC_SUCCESS) {
      std::size_t size = 0;
      n.logSize(program, &size);
      std::string log(size, '\0');
      if (size)
        n.log(program, log.data());
      n.destroy(&program);
      throw std::invalid_argument(std::string("NVRTC compilation failed: ") + n.error(compiled) +
                                  "\n" + log);
    }
    std::size_t size = 0;
    require(n, n.cubinSize(program, &size), "nvrtcGetCUBINSize");
    void *out = std::malloc(size ? size : 1);
    if (!out) {
      n.destroy(&program);
      throw std::runtime_error("out of host memory for the CUBIN");
    }
    const nvrtcResult copied = n.cubin(program, static_cast<char *>(out));
    n.destroy(&program);
    if (copied != NVRTC_SUCCESS) {
      std::free(out);
      require(n, copied, "nvrtcGetCUBIN");
    }
    *binary = out;
    *bytes = size;
    return CKL_OK;
  } catch (const std::invalid_argument &e) {
    ckl::setLastError(e.what());
    return CKL_INVALID_ARGUMENT;
  } catch (const std::exception &e) {
    ckl::setLastError(e.what());
    return CKL_RUNTIME_ERROR;
  }
}

void ckl_binary_free(void *binary) { std::free(binary); }
