// Registry of the sm_100a kernel library linked into libckl_b200.so.
//
// Every entry is a __global__ function whose parameters are the plan's argument slots in
// order: resource pointers, forwarded scalars, and (last) one struct of specialization
// constants passed by value.  The registry records the slot signature so that the runtime
// can validate a committed node before it is launched, and a geometry function that picks
// the grid for given specialization constants.
#pragma once

#include <cstddef>
#include <cstdint>

namespace ckl::library {

struct Geometry {
  unsigned grid[3] = {1, 1, 1};
  unsigned block[3] = {1, 1, 1};
  unsigned sharedBytes = 0;
};

using GeometryFn = bool (*)(const void *spec, std::size_t specBytes, Geometry *out);
// Optional: the __global__ function to launch for given specialization constants, when one
// entry has several compiled tile configurations.
using SelectFn = const void *(*)(const void *spec);

// Optional: bytes of one extra trailing kernel parameter derived from the bound arguments
// (`arguments[i]` points at slot i's bytes, pointers already resolved), e.g. a TMA tensor map
// of a weight buffer.  Returns false when the arguments are invalid for the kernel.
using PrepareFn = bool (*)(const void *spec, const void *const *arguments, std::size_t count,
                           void *extra);

struct Kernel {
  const char *name;
  const void *function;     // host stub of the __global__ function (default configuration)
  const char *signature;    // slot codes: P pointer, I i32, L i64, F f32, D f64, S spec
  std::size_t specBytes;    // size of the trailing specialization struct (0 if none)
  GeometryFn geometry;
  SelectFn select;          // may be null
  PrepareFn prepare = nullptr;
  std::size_t prepareBytes = 0; // size of the parameter `prepare` writes
  // The kernel calls dependentLaunchEntry() first: it may be launched with a programmatic
  // dependency on its predecessors (scheduled while they finish).
  bool dependentLaunch = false;
  // The kernel waits on mbarriers with bounded waits that record a library fault when they
  // expire (ckl_library_faults): the runtime checks the fault word after synchronizing.
  bool boundedWaits = false;
};

// All entries, defined by the kernel translation units (registered at static init time).
const Kernel *find(const char *name);
std::size_t count();
const Kernel *at(std::size_t index);

struct Registrar {
  explicit Registrar(const Kernel &kernel);
};

// Slot size in bytes of one signature code; 0 for an unknown code.
inline std::size_t slotBytes(char code, std::size_t specBytes) {
  switch (code) {
  case 'P': return 8;
  case 'I': return 4;
  case 'L': return 8;
  case 'F': return 4;
  case 'D': return 8;
  case 'S': return specBytes;
  default: return 0;
  }
}

} // namespace ckl::library

#define CKL_CONCAT_INNER(a, b) a##b
#define CKL_CONCAT(a, b) CKL_CONCAT_INNER(a, b)
#define CKL_REGISTER_KERNEL(...)                                                              \
  static const ::ckl::library::Registrar CKL_CONCAT(ckl_registrar_, __LINE__)(                \
      ::ckl::library::Kernel{__VA_ARGS__})
