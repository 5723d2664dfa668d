// Kernel registry: string-named launchers per operator type, filled by static
// initialisers (REGISTER_KERNEL) and looked up by felix::dispatch. Same types
// and macro as the reference (include/felix/registry.hpp:8-34,
// src/felix/base/registry.cpp:7-13). Lookups go through a hash index built on
// insertion instead of a linear scan per call.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace felix {

enum class KernelType : uint8_t { HGEMM, SGEMM, FlashAttn_64, FlashAttn_128, TopK };

struct KernelEntry {
  KernelType type;
  std::string name;
  void* fn_ptr;
  bool stable;
};

class KernelRegistry {
 public:
  void add(KernelEntry k);
  const std::vector<KernelEntry>& all() const;
  // nullptr when (type, name) is not registered.
  const KernelEntry* find(KernelType type, const std::string& name) const;

 private:
  std::vector<KernelEntry> entries;
};

KernelRegistry& global_registry();

}  // namespace felix

#define REGISTER_KERNEL(name, entry)         \
  static bool _##name = []() {               \
    felix::global_registry().add(entry);     \
    return true;                             \
  }()
