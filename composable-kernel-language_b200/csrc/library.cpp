// Registry storage for the sm_100a kernel library (entries register at static init time).
#include "library.hpp"

#include <cstring>
#include <memory>
#include <vector>

namespace ckl::library {
namespace {
std::vector<std::unique_ptr<Kernel>> &storage() {
  static std::vector<std::unique_ptr<Kernel>> entries;
  return entries;
}
} // namespace

Registrar::Registrar(const Kernel &kernel) { storage().push_back(std::make_unique<Kernel>(kernel)); }

const Kernel *find(const char *name) {
  for (const auto &k : storage())
    if (std::strcmp(k->name, name) == 0)
      return k.get();
  return nullptr;
}

std::size_t count() { return storage().size(); }

const Kernel *at(std::size_t index) {
  return index < storage().size() ? storage()[index].get() : nullptr;
}
} // namespace ckl::library
