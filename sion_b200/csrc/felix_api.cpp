// felix:: C++ operator API over the C ABI (felix_c.h): FelixStatus, the kernel
// registry, name-based dispatch and the registered kernel names.
//
// Reference behaviour kept (src/felix/base/felix_api.cpp:7-68,
// src/felix/base/status.cpp:16-49, src/felix/base/registry.cpp:7-13):
//   * every operator dispatches on (KernelType, kernel_name);
//   * an unregistered name throws std::runtime_error("No matching kernel found");
//   * invalid arguments give API_ERROR, launch failures KERNEL_LAUNCH_FAILED;
//   * launches are asynchronous on the caller's stream.
// All reference kernel names are registered and served by the sm_100a kernels:
// the seven SGEMM names by the FFMA kernel (ampere_sgemm_128x128_nn_a1b0 keeps
// its alpha = 1, beta = 0 semantics), the two HGEMM names by the tcgen05 kernel
// with the matching B layout, the flash-attention name by the tcgen05
// attention kernel. New "sm100_*" names are registered alongside.
#include <felix/felix.hpp>
#include <felix/registry.hpp>

#include <sstream>
#include <stdexcept>
#include <type_traits>
#include <unordered_map>

#include "../../include/felix_c.h"

namespace felix {

// ------------------------------------------------------------------ status
FelixStatus::FelixStatus() : type(Type::SUCCESS), cuda_code(cudaSuccess), line(0) {}

FelixStatus::FelixStatus(Type t, cudaError_t code, std::string msg, std::string f, int l,
                         std::string fn)
    : type(t), cuda_code(code), message(std::move(msg)), file(std::move(f)), line(l),
      func(std::move(fn)) {}

bool FelixStatus::ok() const { return type == Type::SUCCESS; }

std::string FelixStatus::str() const {
  if (ok()) return "SUCCESS";
  std::ostringstream oss;
  oss << type_string() << " | cudaError: " << static_cast<int>(cuda_code) << " ("
      << cudaGetErrorString(cuda_code) << ")"
      << " | " << message << " | " << file << ":" << line << " (" << func << ")";
  return oss.str();
}

FelixStatus FelixStatus::make(Type t, cudaError_t code, std::string msg,
                              const std::source_location& loc) {
  return FelixStatus(t, code, std::move(msg), loc.file_name(), static_cast<int>(loc.line()),
                     loc.function_name());
}

const char* FelixStatus::type_string() const {
  switch (type) {
    case Type::SUCCESS: return "SUCCESS";
    case Type::KERNEL_LAUNCH_FAILED: return "KERNEL_LAUNCH_FAILED";
    case Type::KERNEL_RUNTIME_ERROR: return "KERNEL_RUNTIME_ERROR";
    case Type::API_ERROR: return "API_ERROR";
    default: return "UNKNOWN";
  }
}

// ---------------------------------------------------------------- registry
namespace {
struct Key {
  KernelType type;
  std::string name;
  bool operator==(const Key& o) const { return type == o.type && name == o.name; }
};
struct KeyHash {
  size_t operator()(const Key& k) const {
    return std::hash<std::string>()(k.name) * 31u + static_cast<size_t>(k.type);
  }
};
std::unordered_map<Key, size_t, KeyHash>& index() {
  static std::unordered_map<Key, size_t, KeyHash> m;
  return m;
}
}  // namespace

void KernelRegistry::add(KernelEntry k) {
  Key key{k.type, k.name};
  auto it = index().find(key);
  if (it != index().end()) {
    entries[it->second] = std::move(k);  // last registration wins
    return;
  }
  index().emplace(std::move(key), entries.size());
  entries.push_back(std::move(k));
}

const std::vector<KernelEntry>& KernelRegistry::all() const { return entries; }

const KernelEntry* KernelRegistry::find(KernelType type, const std::string& name) const {
  auto it = index().find(Key{type, name});
  return it == index().end() ? nullptr : &entries[it->second];
}

KernelRegistry& global_registry() {
  static KernelRegistry instance;
  return instance;
}

// ---------------------------------------------------------------- dispatch
namespace {

template <typename... Args>
FelixStatus dispatch_kernel(KernelType type, const std::string& name, Args... args) {
  static_assert((!std::is_reference_v<Args> && ...),
                "dispatch_kernel does not allow reference arguments");
  const KernelEntry* k = global_registry().find(type, name);
  if (!k) throw std::runtime_error("No matching kernel found");
  auto fn = reinterpret_cast<FelixStatus (*)(Args...)>(k->fn_ptr);
  return fn(args...);
}

FelixStatus from_c(int code, const std::source_location& loc = std::source_location::current()) {
  if (code == FELIX_SUCCESS) return FelixStatus::success();
  return FelixStatus::make(static_cast<FelixStatus::Type>(code),
                           static_cast<cudaError_t>(felix_last_cuda_error()),
                           felix_last_error_message(), loc);
}

// --- SGEMM launchers (all names share one kernel)
FelixStatus sm100_sgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                        const float* B, float beta, float* C, cudaStream_t stream) {
  return from_c(felix_sgemm(M, N, K, alpha, A, B, beta, C, stream));
}
// ampere_sgemm_128x128_nn_a1b0 computes C = A * B whatever alpha/beta are
// (reference kernels/ampere_sgemm_128x128x16_aligned_wip.cuh:226).
FelixStatus sm100_sgemm_a1b0(uint32_t M, uint32_t N, uint32_t K, float, const float* A,
                             const float* B, float, float* C, cudaStream_t stream) {
  return from_c(felix_sgemm(M, N, K, 1.0f, A, B, 0.0f, C, stream));
}

// --- HGEMM launchers
FelixStatus sm100_hgemm_nn(uint32_t M, uint32_t N, uint32_t K, float alpha, const half* A,
                           const half* B, float beta, half* C, cudaStream_t stream) {
  return from_c(felix_hgemm(M, N, K, alpha, A, B, beta, C, FELIX_B_KN, stream));
}
FelixStatus sm100_hgemm_nt(uint32_t M, uint32_t N, uint32_t K, float alpha, const half* A,
                           const half* B, float beta, half* C, cudaStream_t stream) {
  return from_c(felix_hgemm(M, N, K, alpha, A, B, beta, C, FELIX_B_NK, stream));
}

// --- top-k (k-th value per slice)
FelixStatus sm100_topk(float const* data, float* out, uint32_t num_slices, uint32_t slice_size,
                       uint32_t k, bool largest, cudaStream_t stream) {
  return from_c(felix_topk_select(data, out, num_slices, slice_size, k, largest ? 1 : 0, stream));
}

// --- flash attention launchers
template <int D>
FelixStatus sm100_flash_attn(half* Q, half* K, half* V, half* O, uint32_t heads,
                             uint32_t batch_size, uint32_t seqlen, cudaStream_t stream) {
  return from_c(felix_flash_attn_fwd(Q, K, V, O, nullptr, heads, batch_size, seqlen, D, 0.0f,
                                     stream));
}

}  // namespace

FelixStatus ampere_sgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, float const* A,
                                float const* B, float beta, float* C, cudaStream_t stream,
                                const std::string& kernel_name) {
  return dispatch_kernel(KernelType::SGEMM, kernel_name, M, N, K, alpha, A, B, beta, C, stream);
}

FelixStatus ampere_hgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, half const* A,
                                half const* B, float beta, half* C, cudaStream_t stream,
                                const std::string& kernel_name) {
  return dispatch_kernel(KernelType::HGEMM, kernel_name, M, N, K, alpha, A, B, beta, C, stream);
}

FelixStatus sorting_radix_select_launch(float const* data, float* out, uint32_t num_slices,
                                        uint32_t slice_size, uint32_t k, bool largest,
                                        cudaStream_t stream, const std::string& kernel_name) {
  return dispatch_kernel(KernelType::TopK, kernel_name, data, out, num_slices, slice_size, k,
                         largest, stream);
}

template <>
FelixStatus ampere_flash_attn_launch<64, 64>(half* Q, half* K, half* V, half* O, uint32_t heads,
                                             uint32_t batch_size, uint32_t QKV_seqlen,
                                             cudaStream_t stream, const std::string& kernel_name) {
  return dispatch_kernel(KernelType::FlashAttn_64, kernel_name, Q, K, V, O, heads, batch_size,
                         QKV_seqlen, stream);
}

template <>
FelixStatus ampere_flash_attn_launch<128, 64>(half* Q, half* K, half* V, half* O, uint32_t heads,
                                              uint32_t batch_size, uint32_t QKV_seqlen,
                                              cudaStream_t stream,
                                              const std::string& kernel_name) {
  return dispatch_kernel(KernelType::FlashAttn_128, kernel_name, Q, K, V, O, heads, batch_size,
                         QKV_seqlen, stream);
}

template <>
FelixStatus flash_attn_fwd_lse_launch<64, 64>(half* Q, half* K, half* V, half* O, float* lse,
                                              uint32_t heads, uint32_t batch_size,
                                              uint32_t QKV_seqlen, cudaStream_t stream,
                                              bool causal) {
  return from_c(felix_flash_attn_fwd_ex(Q, K, V, O, lse, heads, batch_size, QKV_seqlen, 64, 0.0f,
                                        causal ? 1 : 0, stream));
}

template <>
FelixStatus flash_attn_fwd_lse_launch<128, 64>(half* Q, half* K, half* V, half* O, float* lse,
                                               uint32_t heads, uint32_t batch_size,
                                               uint32_t QKV_seqlen, cudaStream_t stream,
                                               bool causal) {
  return from_c(felix_flash_attn_fwd_ex(Q, K, V, O, lse, heads, batch_size, QKV_seqlen, 128,
                                        0.0f, causal ? 1 : 0, stream));
}

template <>
FelixStatus flash_attn_bwd_launch<64>(const half* Q, const half* K, const half* V, const half* O,
                                      const half* dO, const float* lse, half* dQ, half* dK,
                                      half* dV, uint32_t heads, uint32_t batch_size,
                                      uint32_t QKV_seqlen, cudaStream_t stream, bool causal) {
  return from_c(felix_flash_attn_bwd(Q, K, V, O, dO, lse, dQ, dK, dV, heads, batch_size,
                                     QKV_seqlen, 64, 0.0f, causal ? 1 : 0, nullptr, 0, stream));
}

template <>
FelixStatus flash_attn_bwd_launch<128>(const half* Q, const half* K, const half* V, const half* O,
                                       const half* dO, const float* lse, half* dQ, half* dK,
                                       half* dV, uint32_t heads, uint32_t batch_size,
                                       uint32_t QKV_seqlen, cudaStream_t stream, bool causal) {
  return from_c(felix_flash_attn_bwd(Q, K, V, O, dO, lse, dQ, dK, dV, heads, batch_size,
                                     QKV_seqlen, 128, 0.0f, causal ? 1 : 0, nullptr, 0, stream));
}

FelixStatus check_watchdog() {
  unsigned code = 0;
  return from_c(felix_watchdog_status(&code, 1));
}

}  // namespace felix

// ------------------------------------------------------------ registrations
#define FELIX_REG(tag, TYPE, NAME, FN, STABLE)                                          \
  REGISTER_KERNEL(tag, (felix::KernelEntry{felix::KernelType::TYPE, NAME,               \
                                           reinterpret_cast<void*>(FN), STABLE}))

FELIX_REG(cute_sgemm_64x64_nn, SGEMM, "cute_sgemm_64x64_nn", &felix::sm100_sgemm, true);
FELIX_REG(cute_sgemm_64x64_nn_swizzle, SGEMM, "cute_sgemm_64x64_nn_swizzle", &felix::sm100_sgemm,
          true);
FELIX_REG(ampere_sgemm_64x64_nn, SGEMM, "ampere_sgemm_64x64_nn", &felix::sm100_sgemm, true);
FELIX_REG(ampere_sgemm_128x128_nn_a1b0, SGEMM, "ampere_sgemm_128x128_nn_a1b0",
          &felix::sm100_sgemm_a1b0, true);
FELIX_REG(cute_sgemm_128x128_nn, SGEMM, "cute_sgemm_128x128_nn", &felix::sm100_sgemm, true);
FELIX_REG(cute_sgemm_128x128_nn_wt, SGEMM, "cute_sgemm_128x128_nn_wt", &felix::sm100_sgemm, true);
FELIX_REG(cute_sgemm_128x128_nn_wt_db, SGEMM, "cute_sgemm_128x128_nn_wt_db", &felix::sm100_sgemm,
          true);
FELIX_REG(sm100_sgemm, SGEMM, "sm100_sgemm", &felix::sm100_sgemm, true);

FELIX_REG(cute_hgemm_128x128_nn, HGEMM, "cute_hgemm_128x128_nn", &felix::sm100_hgemm_nn, true);
FELIX_REG(cute_hgemm_128x128_nt, HGEMM, "cute_hgemm_128x128_nt", &felix::sm100_hgemm_nt, true);
FELIX_REG(sm100_hgemm_nn, HGEMM, "sm100_hgemm_nn", &felix::sm100_hgemm_nn, true);
FELIX_REG(sm100_hgemm_nt, HGEMM, "sm100_hgemm_nt", &felix::sm100_hgemm_nt, true);

FELIX_REG(sorting_radix_select, TopK, "sorting_radix_select", &felix::sm100_topk, true);
FELIX_REG(sm100_topk, TopK, "sm100_topk", &felix::sm100_topk, true);

FELIX_REG(fa64_ampere_name, FlashAttn_64, "ampere_flash_attn_mma16168_64_1D_warp_tiling",
          &felix::sm100_flash_attn<64>, true);
FELIX_REG(fa128_ampere_name, FlashAttn_128, "ampere_flash_attn_mma16168_64_1D_warp_tiling",
          &felix::sm100_flash_attn<128>, true);
FELIX_REG(fa64_sm100, FlashAttn_64, "sm100_flash_attn", &felix::sm100_flash_attn<64>, true);
FELIX_REG(fa128_sm100, FlashAttn_128, "sm100_flash_attn", &felix::sm100_flash_attn<128>, true);
