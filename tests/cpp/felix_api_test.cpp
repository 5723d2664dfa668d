// C++ check of the felix:: operator API in libfelix_b200.so (no GPU needed):
// registry contents, dispatch by (type, name), the unknown-name exception and
// FelixStatus formatting (reference: include/felix/registry.hpp:8-34,
// src/felix/base/felix_api.cpp:7-20, src/felix/base/status.cpp:16-27).
// Exit code 0 = pass; prints one line per failed check.
#include <felix/felix.hpp>
#include <felix/registry.hpp>

#include <cstdio>
#include <set>
#include <stdexcept>
#include <string>

static int failures = 0;
#define CHECK(cond, what)                      \
  do {                                         \
    if (!(cond)) {                             \
      std::printf("FAIL: %s\n", what);         \
      ++failures;                              \
    }                                          \
  } while (0)

int main(int argc, char** argv) {
  const bool have_gpu = argc > 1 && std::string(argv[1]) == "gpu";
  std::set<std::string> names;
  for (const auto& e : felix::global_registry().all()) names.insert(e.name);
  for (const char* n : {"cute_sgemm_64x64_nn", "cute_sgemm_64x64_nn_swizzle", "ampere_sgemm_64x64_nn",
                        "ampere_sgemm_128x128_nn_a1b0", "cute_sgemm_128x128_nn",
                        "cute_sgemm_128x128_nn_wt", "cute_sgemm_128x128_nn_wt_db",
                        "cute_hgemm_128x128_nn", "cute_hgemm_128x128_nt",
                        "ampere_flash_attn_mma16168_64_1D_warp_tiling", "sorting_radix_select",
                        "sm100_sgemm", "sm100_hgemm_nt", "sm100_flash_attn", "sm100_topk"})
    CHECK(names.count(n) == 1, (std::string("registered: ") + n).c_str());
  CHECK(felix::global_registry().find(felix::KernelType::HGEMM, "cute_hgemm_128x128_nt") != nullptr,
        "find HGEMM nt");
  CHECK(felix::global_registry().find(felix::KernelType::SGEMM, "cute_hgemm_128x128_nt") == nullptr,
        "find respects the kernel type");

  // unknown name -> std::runtime_error("No matching kernel found")
  bool threw = false;
  try {
    felix::ampere_sgemm_launch(64, 64, 64, 1.f, nullptr, nullptr, 0.f, nullptr, nullptr, "nope");
  } catch (const std::runtime_error& e) {
    threw = std::string(e.what()) == "No matching kernel found";
  }
  CHECK(threw, "unknown kernel name throws No matching kernel found");

  // invalid arguments are API_ERROR before any device work
  auto st = felix::ampere_hgemm_launch(128, 128, 65, 1.f, nullptr, nullptr, 0.f, nullptr, nullptr,
                                       "cute_hgemm_128x128_nt");
  CHECK(st.type == felix::FelixStatus::Type::API_ERROR, "null operands -> API_ERROR");
  CHECK(st.str().rfind("API_ERROR | cudaError: ", 0) == 0, "FelixStatus::str format");
  st = felix::sorting_radix_select_launch(nullptr, nullptr, 1, 10, 11, true, nullptr);
  CHECK(st.type == felix::FelixStatus::Type::API_ERROR, "topk bad k -> API_ERROR");
  st = felix::sorting_radix_select_launch(nullptr, nullptr, 0, 10, 3, true, nullptr);
  CHECK(st.ok(), "topk zero slices is a no-op");
  CHECK(felix::FelixStatus::success().str() == "SUCCESS", "success str");

  if (!have_gpu) {
    // without a device a real launch reports a status, never throws
    st = felix::ampere_sgemm_launch(64, 64, 64, 1.f, reinterpret_cast<const float*>(16),
                                    reinterpret_cast<const float*>(16), 0.f,
                                    reinterpret_cast<float*>(16), nullptr);
    CHECK(!st.ok(), "no device -> error status");
  }
  if (failures == 0) std::printf("felix_api_test: all checks passed\n");
  return failures == 0 ? 0 : 1;
}
