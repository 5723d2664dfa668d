// C++ check of the felix:: operator API in libfelix_b200.so: registry
// contents, dispatch by (type, name), the unknown-name exception and
// FelixStatus formatting (reference: include/felix/registry.hpp:8-34,
// src/felix/base/felix_api.cpp:7-20, src/felix/base/status.cpp:16-27).
// With the argument "gpu" it also computes through every registered reference
// kernel name (src/felix/base/felix_api.cpp:22-68 of the reference and the
// launchers' REGISTER_KERNEL lines) and compares each result with the fp64 CPU
// oracle (oracle/liboracle.so, linked by the test runner):
// ampere_sgemm_128x128_nn_a1b0 must ignore alpha/beta and compute C = A*B
// (reference kernels/ampere_sgemm_128x128x16_aligned_wip.cuh:226).
// Exit code 0 = pass; prints one line per failed check.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <felix/felix.hpp>
#include <felix/registry.hpp>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

extern "C" {
void oracle_sgemm(int64_t M, int64_t N, int64_t K, double alpha, const float* A, const float* B,
                  double beta, const float* C0, double* out);
void oracle_hgemm(int64_t M, int64_t N, int64_t K, double alpha, const uint16_t* A,
                  const uint16_t* B, int b_layout, double beta, const uint16_t* C0, double* out);
void oracle_attention_rows(int64_t Bn, int64_t H, int64_t S, int64_t D, const uint16_t* Q,
                           const uint16_t* K, const uint16_t* V, double scale,
                           const int64_t* rows, int64_t n_rows, double* O, double* lse,
                           int causal);
void oracle_topk(const uint32_t* data_bits, uint32_t* out_bits, int64_t num_slices,
                 int64_t slice_size, int64_t k, int largest);
}

static int failures = 0;
#define CHECK(cond, what)                      \
  do {                                         \
    if (!(cond)) {                             \
      std::printf("FAIL: %s\n", what);         \
      ++failures;                              \
    }                                          \
  } while (0)

namespace {

// deterministic inputs: a 64-bit LCG mapped to [-1, 1)
struct Lcg {
  uint64_t s;
  float next() {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return float((s >> 40) & 0xffffff) / float(1 << 23) - 1.0f;
  }
};

template <typename T>
T* to_device(const std::vector<T>& h) {
  T* d = nullptr;
  if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
  cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
  return d;
}

template <typename T>
std::vector<T> to_host(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
  return h;
}

double rel_frob(const std::vector<double>& ref, const std::vector<double>& val) {
  double num = 0, den = 0;
  for (size_t i = 0; i < ref.size(); ++i) {
    num += (val[i] - ref[i]) * (val[i] - ref[i]);
    den += ref[i] * ref[i];
  }
  return std::sqrt(num / (den > 0 ? den : 1));
}

double max_abs(const std::vector<double>& ref, const std::vector<double>& val) {
  double m = 0;
  for (size_t i = 0; i < ref.size(); ++i) m = std::fmax(m, std::fabs(val[i] - ref[i]));
  return m;
}

std::vector<uint16_t> half_bits(const std::vector<__half>& h) {
  std::vector<uint16_t> b(h.size());
  std::memcpy(b.data(), h.data(), h.size() * 2);
  return b;
}

std::vector<double> widen(const std::vector<__half>& h) {
  std::vector<double> d(h.size());
  for (size_t i = 0; i < h.size(); ++i) d[i] = __half2float(h[i]);
  return d;
}

void sgemm_names() {
  const uint32_t M = 150, N = 97, K = 131;  // ragged: no tile divides these
  Lcg g{11};
  std::vector<float> A(size_t(M) * K), B(size_t(K) * N), C0(size_t(M) * N);
  for (auto& x : A) x = g.next();
  for (auto& x : B) x = g.next();
  for (auto& x : C0) x = g.next();
  float *dA = to_device(A), *dB = to_device(B), *dC = to_device(C0);
  const float alpha = 0.75f, beta = -0.5f;
  std::vector<double> ref(size_t(M) * N), ref_a1b0(size_t(M) * N);
  oracle_sgemm(M, N, K, alpha, A.data(), B.data(), beta, C0.data(), ref.data());
  oracle_sgemm(M, N, K, 1.0, A.data(), B.data(), 0.0, nullptr, ref_a1b0.data());
  for (const char* name : {"cute_sgemm_64x64_nn", "cute_sgemm_64x64_nn_swizzle",
                           "ampere_sgemm_64x64_nn", "ampere_sgemm_128x128_nn_a1b0",
                           "cute_sgemm_128x128_nn", "cute_sgemm_128x128_nn_wt",
                           "cute_sgemm_128x128_nn_wt_db", "sm100_sgemm"}) {
    cudaMemcpy(dC, C0.data(), C0.size() * 4, cudaMemcpyHostToDevice);
    auto st = felix::ampere_sgemm_launch(M, N, K, alpha, dA, dB, beta, dC, nullptr, name);
    cudaDeviceSynchronize();
    CHECK(st.ok(), (std::string("sgemm launch ok: ") + name).c_str());
    auto out = to_host(dC, C0.size());
    std::vector<double> o(out.begin(), out.end());
    const bool a1b0 = std::string(name) == "ampere_sgemm_128x128_nn_a1b0";
    const double rf = rel_frob(a1b0 ? ref_a1b0 : ref, o);
    if (!(rf <= 1e-5)) std::printf("  %s rel_frob %.3e\n", name, rf);
    CHECK(rf <= 1e-5, (std::string("sgemm result vs oracle: ") + name).c_str());
  }
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
}

void hgemm_names() {
  const uint32_t M = 200, N = 136, K = 264;
  Lcg g{12};
  std::vector<__half> A(size_t(M) * K), B(size_t(N) * K), C0(size_t(M) * N);
  for (auto& x : A) x = __float2half(g.next());
  for (auto& x : B) x = __float2half(g.next());
  for (auto& x : C0) x = __float2half(g.next());
  const float alpha = 0.5f, beta = 0.25f;
  half *dA = to_device(A), *dB = to_device(B), *dC = to_device(C0);
  for (const char* name : {"cute_hgemm_128x128_nn", "cute_hgemm_128x128_nt", "sm100_hgemm_nn",
                           "sm100_hgemm_nt"}) {
    const bool nt = std::string(name).find("_nt") != std::string::npos;
    // the same B buffer read as [N x K] ("nt") or [K x N] ("nn")
    std::vector<double> ref(size_t(M) * N);
    oracle_hgemm(M, N, K, alpha, half_bits(A).data(), half_bits(B).data(), nt ? 1 : 0, beta,
                 half_bits(C0).data(), ref.data());
    cudaMemcpy(dC, C0.data(), C0.size() * 2, cudaMemcpyHostToDevice);
    auto st = felix::ampere_hgemm_launch(M, N, K, alpha, dA, dB, beta, dC, nullptr, name);
    cudaDeviceSynchronize();
    CHECK(st.ok(), (std::string("hgemm launch ok: ") + name).c_str());
    auto o = widen(to_host(dC, C0.size()));
    const double rf = rel_frob(ref, o);
    double worst = 0;  // per element: |err| <= max(1e-2, 1 fp16 ulp of |ref|)
    for (size_t i = 0; i < ref.size(); ++i) {
      const double a = std::fmax(std::fabs(ref[i]), 6.103515625e-05);
      const double ulp = std::ldexp(1.0, int(std::floor(std::log2(a))) - 10);
      worst = std::fmax(worst, std::fabs(o[i] - ref[i]) / std::fmax(1e-2, ulp));
    }
    if (!(rf <= 1e-3 && worst <= 1.0)) std::printf("  %s rel_frob %.3e worst %.3f\n", name, rf, worst);
    CHECK(rf <= 1e-3 && worst <= 1.0, (std::string("hgemm result vs oracle: ") + name).c_str());
  }
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
}

template <int D>
void attention_names() {
  const uint32_t Bn = 2, H = 3, S = 192;
  const size_t n = size_t(Bn) * H * S * D;
  Lcg g{13 + D};
  std::vector<__half> Q(n), K(n), V(n);
  for (auto* t : {&Q, &K, &V})
    for (auto& x : *t) x = __float2half(2.0f * g.next());
  std::vector<double> ref(n), lse(size_t(Bn) * H * S);
  oracle_attention_rows(Bn, H, S, D, half_bits(Q).data(), half_bits(K).data(), half_bits(V).data(),
                        0.0, nullptr, 0, ref.data(), lse.data(), 0);
  half *dQ = to_device(Q), *dK = to_device(K), *dV = to_device(V), *dO = nullptr;
  cudaMalloc(&dO, n * 2);
  for (const char* name : {"ampere_flash_attn_mma16168_64_1D_warp_tiling", "sm100_flash_attn"}) {
    cudaMemset(dO, 0xff, n * 2);  // NaN pattern: every element must be written
    auto st = felix::ampere_flash_attn_launch<D, 64>(dQ, dK, dV, dO, H, Bn, S, nullptr, name);
    cudaDeviceSynchronize();
    CHECK(st.ok(), (std::string("attention launch ok: ") + name).c_str());
    auto o = widen(to_host(dO, n));
    const double ma = max_abs(ref, o), rf = rel_frob(ref, o);
    if (!(ma <= 1e-2 && rf <= 1e-3)) std::printf("  %s D=%d max_abs %.3e rel_frob %.3e\n", name, D, ma, rf);
    CHECK(ma <= 1e-2 && rf <= 1e-3, (std::string("attention result vs oracle: ") + name).c_str());
  }
  cudaFree(dQ);
  cudaFree(dK);
  cudaFree(dV);
  cudaFree(dO);
}

void topk_names() {
  const uint32_t slices = 5, size = 3000, k = 1000;
  Lcg g{14};
  std::vector<float> x(size_t(slices) * size);
  for (auto& v : x) v = g.next() * 100.f;
  std::vector<uint32_t> bits(x.size()), ref(slices);
  std::memcpy(bits.data(), x.data(), x.size() * 4);
  float* dx = to_device(x);
  float* dout = nullptr;
  cudaMalloc(&dout, slices * 4);
  for (bool largest : {true, false}) {
    oracle_topk(bits.data(), ref.data(), slices, size, k, largest ? 1 : 0);
    for (const char* name : {"sorting_radix_select", "sm100_topk"}) {
      auto st = felix::sorting_radix_select_launch(dx, dout, slices, size, k, largest, nullptr, name);
      cudaDeviceSynchronize();
      CHECK(st.ok(), (std::string("topk launch ok: ") + name).c_str());
      auto o = to_host(dout, slices);
      CHECK(std::memcmp(o.data(), ref.data(), slices * 4) == 0,
            (std::string("topk bit-exact vs oracle: ") + name).c_str());
    }
  }
  cudaFree(dx);
  cudaFree(dout);
}

void gpu_checks() {
  sgemm_names();
  hgemm_names();
  attention_names<64>();
  attention_names<128>();
  topk_names();
  CHECK(felix::check_watchdog().ok(), "watchdog clear after the named launches");
}

}  // namespace

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
  if (have_gpu) gpu_checks();
  if (failures == 0) std::printf("felix_api_test: all checks passed\n");
  return failures == 0 ? 0 : 1;
}
