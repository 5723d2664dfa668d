// Internal host-side interfaces shared by the kernel translation units and the
// C-ABI layer (felix_c.cu). Nothing here is exported.
#pragma once
#include <atomic>
#include <mutex>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "../../include/felix_c.h"

namespace felix_impl {

struct FelixCode {
  int type;          // FELIX_SUCCESS / FELIX_KERNEL_LAUNCH_FAILED / ... (felix_c.h)
  cudaError_t cuda;  // underlying CUDA error, cudaSuccess if none
};

// Record a message for felix_last_error_message() and return the code.
FelixCode api_error(const char* msg, cudaError_t e = cudaErrorInvalidValue);
FelixCode launch_error(cudaError_t e, const char* msg);

struct DeviceInfo {
  int ordinal;
  int num_sms;
  int max_smem_optin;
  unsigned* status_word;  // device address of the watchdog word
};

// One-time, per-device set-up (kernel attributes and the like), safe to call
// from several host threads: the first caller on a device runs `setup`
// (returning 0 on success) under a lock; later calls see the flag without
// locking. A failed set-up is retried on the next call.
class PerDeviceOnce {
 public:
  template <class F>
  int run(int device, F&& setup) {
    if (device < 0 || device >= 64) return -1;
    if (done_[device].load(std::memory_order_acquire)) return 0;
    std::lock_guard<std::mutex> lk(mu_);
    if (done_[device].load(std::memory_order_relaxed)) return 0;
    const int rc = setup();
    if (rc == 0) done_[device].store(true, std::memory_order_release);
    return rc;
  }

 private:
  std::mutex mu_;
  std::atomic<bool> done_[64] = {};
};

// Per-device facts for the current device (initialised once per device).
DeviceInfo* current_device_info();

// Scratch layout shared by every kernel that uses a workspace: a fixed block
// of kWsMaxCounters 32-bit tile counters at offset 0 (always left at zero by
// the kernels), then the fp32 partial tiles. Keeping the counters at a fixed
// place lets operators share one buffer without clobbering each other's
// zero invariant.
constexpr size_t kWsCounterBytes = 16384;
constexpr uint32_t kWsMaxCounters = kWsCounterBytes / 4;

// Library-owned scratch for a (device, stream) pair, grown on demand and
// zero-filled on (re)allocation. Kernels leave their counters at zero.
void* library_workspace(DeviceInfo* dev, cudaStream_t stream, size_t bytes);

// 2-D fp16 tensor map, 128-byte swizzle: inner extent `inner` elements,
// `outer` rows, row pitch in bytes, box of box_inner x box_outer.
int encode_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer);
// 2-D fp16 tensor map with an explicit swizzle span (0, 32, 64 or 128 bytes).
int encode_tmap_2d_f16_swizzle(CUtensorMap* map, const void* base, uint64_t inner,
                               uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner,
                               uint32_t box_outer, int swizzle_bytes);
// 3-D fp16 tensor map, 128-byte swizzle: [outer2][outer1][inner].
int encode_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer1,
                       uint64_t outer2, uint64_t pitch1_bytes, uint64_t pitch2_bytes,
                       uint32_t box_inner, uint32_t box_outer1, uint32_t box_outer2);
// 2-D fp32 tensor map (row pitch in bytes, multiple of 16), unswizzled or with
// the 128-byte swizzle (box_inner * 4 must then be 128).
int encode_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                       bool swizzle128 = false);
// 3-D fp32 tensor map, 128-byte swizzle (box_inner * 4 must be <= 128).
int encode_tmap_3d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer1,
                       uint64_t outer2, uint64_t pitch1_bytes, uint64_t pitch2_bytes,
                       uint32_t box_inner, uint32_t box_outer1, uint32_t box_outer2);
// Same without swizzle (used for plain row stores / loads).
int encode_tmap_2d_f16_noswizzle(CUtensorMap* map, const void* base, uint64_t inner,
                                 uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner,
                                 uint32_t box_outer);

FelixCode scale_half_matrix(__half* C, size_t n, float beta, cudaStream_t stream);
FelixCode scale_float_matrix(float* C, size_t n, float beta, cudaStream_t stream);

struct HgemmOptions {
  int block_n = 0;   // 0 = auto, 64, 128 or 256
  int stream_k = 0;  // 0 = auto, 1 = off, 2 = on whenever the last wave is partial
  int max_ctas = 0;  // 0 = one per SM; otherwise cap the persistent grid
  int cta_pair = 0;  // 0 = auto (pairs for large shapes), 1 = off, 2 = CTA pairs (cta_group::2)
};

size_t hgemm_workspace_bytes(uint32_t M, uint32_t N, uint32_t K, const HgemmOptions& o,
                             int num_sms);
FelixCode hgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, const __half* A,
                       const __half* B, float beta, __half* C, bool b_kn, const HgemmOptions& o,
                       void* workspace, size_t ws_bytes, cudaStream_t stream);

struct SgemmOptions {
  int split_k = 0;             // 0 = auto, 1 = none, n = n-way
  bool allow_stream_k = true;  // auto may pick stream-K (workspace grows with the SM count)
  bool allow_tma = true;       // TMA-fed main loop when rows are 16-byte aligned
  bool forbid_alloc = false;   // never fall back to the library workspace (allocation-free callers)
};
size_t sgemm_workspace_bytes(uint32_t M, uint32_t N, uint32_t K, const SgemmOptions& o,
                             int num_sms);
FelixCode sgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                       const float* B, float beta, float* C, const SgemmOptions& o,
                       void* workspace, size_t ws_bytes, cudaStream_t stream);

FelixCode sgemm_noalloc_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                               const float* B, float beta, float* C, int split_k,
                               cudaStream_t stream);

FelixCode flash_attn_launch(const __half* Q, const __half* K, const __half* V, __half* O,
                            float* lse, uint32_t heads, uint32_t batch, uint32_t seqlen,
                            uint32_t head_dim, float scale, bool causal, cudaStream_t stream);

size_t flash_attn_bwd_workspace_bytes(uint32_t heads, uint32_t batch, uint32_t seqlen,
                                      uint32_t head_dim);
FelixCode flash_attn_bwd_launch(const __half* Q, const __half* K, const __half* V,
                                const __half* O, const __half* dO, const float* lse, __half* dQ,
                                __half* dK, __half* dV, uint32_t heads, uint32_t batch,
                                uint32_t seqlen, uint32_t head_dim, float scale, bool causal,
                                void* workspace, size_t ws_bytes, cudaStream_t stream);

FelixCode topk_select_launch(const float* data, float* out, uint32_t num_slices,
                             uint32_t slice_size, uint32_t k, bool largest, cudaStream_t stream);

FelixCode watchdog_probe_launch(uint32_t limit_us, cudaStream_t stream);

}  // namespace felix_impl
