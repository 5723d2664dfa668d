// C entry points into the reference's own operator library (Aoi979/Sion, built
// unmodified from its sources by oracle/build_ref.sh into oracle/_ref/) —
// TEST INFRASTRUCTURE ONLY: used by tests/ and bench.py's reference comparator
// to run the reference's kernels on the same seeded inputs, never by the
// product path. Calls go through the reference's felix:: API with the kernel
// names its own sion:: wrappers use (reference src/sion/gemm/sgemm/sgemm.cpp:26,
// src/sion/gemm/hgemm/hgemm.cpp:33-37,75-78, src/sion/flash_attention/flash_attn.cpp:34-36).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <felix/felix.hpp>

#include <cstdint>
#include <exception>

extern "C" {

int ref_sgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A, const float* B,
              float beta, float* C, void* stream) {
  try {
    return static_cast<int>(felix::ampere_sgemm_launch(M, N, K, alpha, A, B, beta, C,
                                                       static_cast<cudaStream_t>(stream),
                                                       "cute_sgemm_64x64_nn")
                                .type);
  } catch (const std::exception&) {
    return -1;
  }
}

// nt != 0: B stored N x K ("cute_hgemm_128x128_nt"), else K x N ("_nn").
int ref_hgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A, const void* B,
              float beta, void* C, int nt, void* stream) {
  try {
    return static_cast<int>(
        felix::ampere_hgemm_launch(M, N, K, alpha, static_cast<const half*>(A),
                                   static_cast<const half*>(B), beta, static_cast<half*>(C),
                                   static_cast<cudaStream_t>(stream),
                                   nt ? "cute_hgemm_128x128_nt" : "cute_hgemm_128x128_nn")
            .type);
  } catch (const std::exception&) {
    return -1;
  }
}

int ref_flash_attn(void* Q, void* K, void* V, void* O, uint32_t heads, uint32_t batch,
                   uint32_t seqlen, uint32_t head_dim, void* stream) {
  try {
    half *q = static_cast<half*>(Q), *k = static_cast<half*>(K), *v = static_cast<half*>(V),
         *o = static_cast<half*>(O);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (head_dim == 128)
      return static_cast<int>(
          felix::ampere_flash_attn_launch<128, 64>(q, k, v, o, heads, batch, seqlen, s).type);
    if (head_dim == 64)
      return static_cast<int>(
          felix::ampere_flash_attn_launch<64, 64>(q, k, v, o, heads, batch, seqlen, s).type);
    return -2;
  } catch (const std::exception&) {
    return -1;
  }
}

}  // extern "C"
