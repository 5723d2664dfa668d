// felix operator API (libfelix_b200.so). The four entry points keep the
// reference's exact signatures and default kernel names
// (include/felix/felix.hpp:7-28 of the reference); the named kernels are served
// by the sm_100a kernels of this library. Additions are marked "new".
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <felix/status.hpp>
#include <string>

namespace felix {

FelixStatus ampere_sgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, float const* A,
                                float const* B, float beta, float* C, cudaStream_t stream,
                                const std::string& kernel_name = "cute_sgemm_64x64_nn");

FelixStatus ampere_hgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, half const* A,
                                half const* B, float beta, half* C, cudaStream_t stream,
                                const std::string& kernel_name = "cute_hgemm_128x128_nn");

// k-th largest / smallest value per slice ("sorting_radix_select" and
// "sm100_topk" both select the sm_100a radix-select kernels).
FelixStatus sorting_radix_select_launch(float const* data, float* out, uint32_t num_slices,
                                        uint32_t slice_size, uint32_t k, bool largest,
                                        cudaStream_t stream,
                                        const std::string& kernel_name = "sorting_radix_select");

template <int HEAD_DIM, int Bc = 64>
FelixStatus ampere_flash_attn_launch(half* Q, half* K, half* V, half* O, uint32_t heads,
                                     uint32_t batch_size, uint32_t QKV_seqlen,
                                     cudaStream_t stream,
                                     const std::string& kernel_name =
                                         "ampere_flash_attn_mma16168_64_1D_warp_tiling");

// new: same operator with the fp32 natural-log LSE of every query row
// ([batch, heads, seqlen]; lse may be nullptr) and an optional causal mask
// (query i attends to keys 0..i).
template <int HEAD_DIM, int Bc = 64>
FelixStatus flash_attn_fwd_lse_launch(half* Q, half* K, half* V, half* O, float* lse,
                                      uint32_t heads, uint32_t batch_size, uint32_t QKV_seqlen,
                                      cudaStream_t stream, bool causal = false);

// new: attention backward. Given Q, K, V, the forward output O and its LSE
// (from flash_attn_fwd_lse_launch) and dO, writes dQ, dK, dV (all fp16
// [batch, heads, seqlen, HEAD_DIM]). Library-owned fp32 scratch (dQ
// accumulator, per-row dO.O) is allocated on first use per device and stream.
// No reference counterpart: the reference has a forward operator only.
template <int HEAD_DIM>
FelixStatus flash_attn_bwd_launch(const half* Q, const half* K, const half* V, const half* O,
                                  const half* dO, const float* lse, half* dQ, half* dK, half* dV,
                                  uint32_t heads, uint32_t batch_size, uint32_t QKV_seqlen,
                                  cudaStream_t stream, bool causal = false);

// new: reads (and clears) the device watchdog word; KERNEL_RUNTIME_ERROR when a
// bounded wait inside a kernel gave up. Synchronises the device.
FelixStatus check_watchdog();

}  // namespace felix
