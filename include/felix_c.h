/*
 * felix_c.h — C ABI of the sm_100a operator library (libfelix_b200.so).
 *
 * Plain pointers, sizes and an opaque stream handle (a cudaStream_t passed as
 * void*; NULL = legacy default stream). No C++ or torch types cross this
 * boundary. All device pointers are caller-owned; launches are asynchronous on
 * the given stream and never synchronise. Every function returns a status
 * type code that maps 1:1 onto felix::FelixStatus::Type
 * (reference: include/felix/status.hpp:10-15); the CUDA error behind a failure
 * and a readable message are kept per calling thread.
 *
 * fp16 data is passed as `const void*` / `void*` holding IEEE binary16 values.
 */
#ifndef FELIX_C_H
#define FELIX_C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status type codes (== felix::FelixStatus::Type, include/felix/status.hpp:10-15). */
#define FELIX_SUCCESS 0
#define FELIX_KERNEL_LAUNCH_FAILED 1
#define FELIX_KERNEL_RUNTIME_ERROR 2
#define FELIX_API_ERROR 3

/* B operand storage for HGEMM. */
#define FELIX_B_KN 0 /* "nn": B stored K x N row-major (cute_hgemm_128x128_nn)        */
#define FELIX_B_NK 1 /* "nt": B stored N x K row-major, i.e. column-major K x N (_nt) */

/* CUDA error code behind the last non-success status on this thread (0 if none). */
int felix_last_cuda_error(void);
/* Human-readable message for the last non-success status on this thread. */
const char* felix_last_error_message(void);
/* Library version string. */
const char* felix_version(void);

/*
 * SGEMM, fp32 SIMT: C = alpha * A * B + beta * C.
 * A [M x K], B [K x N], C [M x N], all row-major fp32.
 * Replaces felix::ampere_sgemm_launch (reference include/felix/felix.hpp:7-10,
 * src/felix/base/felix_api.cpp:22-28; default kernel cute_sgemm_64x64_nn,
 * src/felix/gemm/sgemm/cute_sgemm_64x64_nn_kernel_launch.cu:7-63).
 * Any M, N, K (no alignment requirement). beta == 0 never reads C.
 */
int felix_sgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                const float* B, float beta, float* C, void* stream);

/*
 * SGEMM with explicit split-K and caller-owned workspace.
 * split_k: 0 = auto, 1 = none, n = n-way. workspace may be NULL (library-owned
 * per-stream scratch); otherwise it must hold felix_sgemm_workspace_size()
 * bytes and be zero-filled before its first use (the kernel leaves its
 * counters at zero). No reference counterpart: the reference has no split-K.
 */
int felix_sgemm_ex(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                   const float* B, float beta, float* C, int split_k, void* workspace,
                   size_t workspace_bytes, void* stream);
int felix_sgemm_workspace_size(uint32_t M, uint32_t N, uint32_t K, int split_k,
                               size_t* bytes);

/*
 * SGEMM that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc from inside an operator call: hosts
 * that own all device memory through their own pool or a fixed memory budget,
 * plugin runtimes that forbid allocation in a kernel launch path, and
 * latency-critical code that cannot accept cudaMalloc's implicit device-wide
 * synchronisation. Same arithmetic and arguments as felix_sgemm_ex; the
 * split-K scratch (tile counters + fp32 partial tiles) lives in a static
 * array inside the library's device image instead of being allocated:
 *   - size: 16 MiB of partial tiles + 16 KiB of counters, held by every GPU
 *     that loads the library until the process exits;
 *   - split_k = 0 picks the largest automatic split whose partials fit;
 *     an explicit split_k > 1 with tiles x split_k > 256 (tiles =
 *     ceil(M/128) * ceil(N/128); checked on the requested split_k, before
 *     it is clamped to ceil(K/16)) is rejected with FELIX_API_ERROR;
 *   - it never falls back to an allocated workspace: a scratch that does not
 *     fit is an FELIX_API_ERROR, not a cudaMalloc;
 *   - the first call on a device looks up the scratch's device address
 *     (cudaGetSymbolAddress) for that device; make that first call before any
 *     stream capture;
 *   - each call clears the counters on `stream` before its kernel;
 *   - all calls share the one array: calls whose execution overlaps on the GPU
 *     (different streams without ordering) race and give wrong results.
 * The caller still owns A, B and C.
 */
int felix_sgemm_noalloc(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                        const float* B, float beta, float* C, int split_k, void* stream);

/*
 * HGEMM, fp16 tensor cores (tcgen05, fp32 accumulate in TMEM, fp16 output):
 * C = alpha * A * op(B) + beta * C. A [M x K] row-major; B per b_layout
 * (FELIX_B_KN or FELIX_B_NK); C [M x N] row-major.
 * Replaces felix::ampere_hgemm_launch with kernel names "cute_hgemm_128x128_nn"
 * / "cute_hgemm_128x128_nt" (reference include/felix/felix.hpp:12-15,
 * src/felix/base/felix_api.cpp:30-36,
 * src/felix/gemm/hgemm/cute_hgemm_128x128_{nn,nt}_kernel_launch.cu).
 * The reference accumulates in fp16; this accumulates in fp32.
 * Requirements: K % 8 == 0; for FELIX_B_KN also N % 8 == 0; A, B 16-byte
 * aligned (C too when N % 8 == 0). M, N, K need not be tile multiples
 * (the reference requires M, N % 128 and K % 64).
 */
int felix_hgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A, const void* B,
                float beta, void* C, int b_layout, void* stream);

/*
 * HGEMM with explicit schedule and caller-owned workspace (no reference
 * counterpart; the reference has no split-K / stream-K).
 * block_n: 0 auto, 64, 128 or 256. stream_k: 0 auto, 1 off, 2 on whenever the last
 * wave of tiles is incomplete. max_ctas: 0 = one persistent CTA per SM.
 * workspace: NULL = library-owned per-(device, stream) scratch; otherwise at
 * least felix_hgemm_workspace_size() bytes, zero-filled before first use. Its
 * first 16 KiB are counters (stream-K tickets; for shapes of four or more
 * waves of tiles, the counter that hands whole tiles out at run time) that
 * every launch leaves at zero, so launches that share a workspace must not
 * overlap on the GPU.
 */
int felix_hgemm_ex(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A,
                   const void* B, float beta, void* C, int b_layout, int block_n, int stream_k,
                   int max_ctas, void* workspace, size_t workspace_bytes, void* stream);
int felix_hgemm_workspace_size(uint32_t M, uint32_t N, uint32_t K, int block_n, int stream_k,
                               int max_ctas, size_t* bytes);
/*
 * felix_hgemm_ex plus cta_pair (no reference counterpart): 0 auto (pairs when
 * M, N >= 256, K >= 512 with K (and N for FELIX_B_KN) a multiple of 64, and at
 * least one wave of 256 x 256 tiles, with block_n, stream_k, max_ctas all 0),
 * 1 off, 2 = 256 x 256 tiles computed by 2-CTA clusters with cta_group::2 MMAs
 * (each CTA loads its 128 rows of A and half of the tile's B, the leader
 * issues M = 256 MMAs; block_n must be 0 or 256; K, and N for FELIX_B_KN,
 * multiples of 64). felix_hgemm and felix_hgemm_ex use the same automatic
 * choice. Workspace size from felix_hgemm_workspace_size2 with the same
 * options.
 */
int felix_hgemm_ex2(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A,
                    const void* B, float beta, void* C, int b_layout, int block_n, int stream_k,
                    int max_ctas, int cta_pair, void* workspace, size_t workspace_bytes,
                    void* stream);
int felix_hgemm_workspace_size2(uint32_t M, uint32_t N, uint32_t K, int block_n, int stream_k,
                                int max_ctas, int cta_pair, size_t* bytes);

/*
 * Flash-attention forward, fp16, no mask: O = softmax(Q K^T * scale) V per
 * (batch, head). Q, K, V, O are [batch, heads, seqlen, head_dim] contiguous
 * fp16. lse (optional, may be NULL) receives the fp32 natural-log
 * log-sum-exp of each query row, [batch, heads, seqlen].
 * scale <= 0 selects the reference's fixed 1/sqrt(head_dim).
 * Replaces felix::ampere_flash_attn_launch<HEAD_DIM, 64> (reference
 * include/felix/felix.hpp:22-28, src/felix/base/felix_api.cpp:47-68,
 * src/felix/flash_attention/ampere_flash_attn_mma16168_64_1D_warp_tiling_kernel_launch.cu:8-55),
 * which supports head_dim 64/128 and seqlen % 64 == 0 and has no LSE output.
 * Here: head_dim in {64, 128}, any seqlen >= 1.
 */
int felix_flash_attn_fwd(const void* Q, const void* K, const void* V, void* O, float* lse,
                         uint32_t heads, uint32_t batch, uint32_t seqlen, uint32_t head_dim,
                         float scale, void* stream);

/*
 * Flash-attention forward with an optional causal mask (causal != 0: query i
 * attends to keys 0..i, queries and keys aligned at position 0, as
 * scaled_dot_product_attention(is_causal=True) with equal lengths). Otherwise
 * identical to felix_flash_attn_fwd. No reference counterpart: the reference
 * kernel supports no mask (reference README.md:23).
 */
int felix_flash_attn_fwd_ex(const void* Q, const void* K, const void* V, void* O, float* lse,
                            uint32_t heads, uint32_t batch, uint32_t seqlen, uint32_t head_dim,
                            float scale, int causal, void* stream);

/*
 * Flash-attention backward (no reference counterpart; the reference has a
 * forward kernel only): given Q, K, V, the forward output O, its gradient dO
 * (all fp16 [batch, heads, seqlen, head_dim]) and the forward's fp32
 * natural-log LSE [batch, heads, seqlen], writes dQ, dK, dV (fp16, same
 * shape). scale <= 0 selects 1/sqrt(head_dim); causal as in
 * felix_flash_attn_fwd_ex. workspace: NULL = library-owned scratch, else at
 * least felix_flash_attn_bwd_workspace_size() bytes (fp32 dQ accumulator and
 * the per-row dO.O sums; its contents need no initialisation).
 */
int felix_flash_attn_bwd(const void* Q, const void* K, const void* V, const void* O,
                         const void* dO, const float* lse, void* dQ, void* dK, void* dV,
                         uint32_t heads, uint32_t batch, uint32_t seqlen, uint32_t head_dim,
                         float scale, int causal, void* workspace, size_t workspace_bytes,
                         void* stream);
int felix_flash_attn_bwd_workspace_size(uint32_t heads, uint32_t batch, uint32_t seqlen,
                                        uint32_t head_dim, size_t* bytes);

/*
 * k-th value per slice (radix select): out[s] = the k-th largest (largest != 0)
 * or k-th smallest value of data[s * slice_size, (s + 1) * slice_size), fp32,
 * returned bit-exactly (order: NaN above +inf, -0.0 below +0.0).
 * Replaces felix::sorting_radix_select_launch / "sorting_radix_select"
 * (reference include/felix/felix.hpp:17-20,
 * src/felix/topk/sorting_radix_select_kernel_launch.cu:7-38); same argument
 * rules: num_slices == 0 is a no-op, null pointers or k outside
 * [1, slice_size] are FELIX_API_ERROR.
 */
int felix_topk_select(const float* data, float* out, uint32_t num_slices, uint32_t slice_size,
                      uint32_t k, int largest, void* stream);

/*
 * Device watchdog. Every bounded wait inside the kernels records a nonzero
 * site code in a per-device status word when it gives up. Reads (and, when
 * clear != 0, resets) the word of the current device; synchronises the device.
 * Returns FELIX_KERNEL_RUNTIME_ERROR when the word was nonzero.
 */
int felix_watchdog_status(unsigned* code, int clear);

/*
 * Test hook for the watchdog: launches one CTA that waits on an mbarrier no
 * one arrives on, with a limit of limit_us microseconds (1..1000000). The wait
 * gives up, records its site code and the kernel returns normally.
 */
int felix_watchdog_probe(uint32_t limit_us, void* stream);

/* Number of SMs of the current device (persistent grid size). */
int felix_num_sms(int* count);

#ifdef __cplusplus
}
#endif

#endif /* FELIX_C_H */
