// SGEMM for sm_100a on the FP32 FFMA pipe: C = alpha * A * B + beta * C,
// A [M x K], B [K x N], C [M x N] row-major fp32.
// Replaces the SIMT kernels behind felix::ampere_sgemm_launch (reference:
// src/felix/gemm/sgemm/cute_sgemm_64x64_nn_kernel_launch.cu:7-63 and
// kernels/cute_ampere_sgemm_64x64_nn.cuh:9-224, default "cute_sgemm_64x64_nn";
// the other six registered SGEMM names route here too).
//
// Design: 128 x 128 CTA tile, 256 threads, each thread an 8 x 8 register block
// (two 4-wide row groups x two 4-wide column groups, so shared-memory reads are
// 128-bit and conflict-free), K step 16 (8 builds too), double-buffered shared
// memory fed by 128-bit global loads staged in registers (one barrier per K
// step), operand fragments double-buffered in registers. Measured on B200
// (1024^3 / 4096^3 TFLOP/s): BK 16 + 2 CTAs/SM 29.9 / 44.7, BK 8 + 2 CTAs/SM
// 28.3 / 42.3; a packed fma.rn.f32x2 inner product was slower (25.0 / 38.7),
// and so was an 8 x 16 register block with a 128 x 256 tile (16.4 / 33.5). Any M, N, K:
// loads are predicated with zero fill, stores are bounds-checked; the 128-bit
// path is used when rows are 16-byte aligned. When the tiles do not fill one
// wave of two CTAs per SM (e.g. 1024^3: 64 tiles), the automatic
// schedule is stream-K: 2 x SMs CTAs take equal runs of (tile, k-tile)
// iterations; an explicit split count splits along K instead. Either way the
// last CTA of a tile to finish (atomic ticket) sums the fp32 partials in a
// fixed order — deterministic, and no CTA waits on another.
// Few tiles with short K per split instead form clusters of S K-splits per
// tile that sum their partials through distributed shared memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

#include "felix_internal.h"
#include "sm100_ptx.cuh"

namespace felix_sm100 {
namespace sgemm {

#ifdef FELIX_SGEMM_TRACE
// Development-only per-CTA timeline (compiled out of the library build):
// [cta][event] = globaltimer ns.
__device__ unsigned long long g_sg_trace[1024][8];
#define SG_TR(ev)                                                          \
  do {                                                                     \
    const unsigned b_ = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x; \
    if (threadIdx.x == 0 && b_ < 1024) {                                   \
      unsigned long long t_;                                               \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                \
      g_sg_trace[b_][ev] = t_;                                             \
    }                                                                      \
  } while (0)
#else
#define SG_TR(ev) \
  do {            \
  } while (0)
#endif

#ifndef FELIX_SGEMM_BK
#define FELIX_SGEMM_BK 16
#endif
#ifndef FELIX_SGEMM_MINB
#define FELIX_SGEMM_MINB 2
#endif
#ifndef FELIX_SGEMM_TN
#define FELIX_SGEMM_TN 8
#endif
// Per-thread register block 8 x TN (TN = 8: CTA tile 128 x 128; TN = 16: 128 x 256).
constexpr int TN = FELIX_SGEMM_TN;
constexpr int NB = TN / 4;  // 4-wide column groups per thread, 64 columns apart
constexpr int BM = 128, BN = 16 * TN, BK = FELIX_SGEMM_BK, kThreads = 256;
constexpr int kLd = BK / 8;             // float4 loads of A per thread per k-tile
constexpr int kLdB = BN * BK / 1024;    // float4 loads of B per thread per k-tile
constexpr int kPartF4 = 2 * TN;         // float4s of a thread's partial block
static_assert(TN == 8 || TN == 16, "register block");
static_assert(BK == 8 || BK == 16, "k-tile");
constexpr int APAD = 4;  // As row pitch 132 floats: transposed stores avoid bank conflicts

struct Params {
  uint32_t M, N, K;
  float alpha, beta;
  const float* A;
  const float* B;
  float* C;
  uint32_t splits, k_per_split;  // k_per_split is a multiple of BK
  uint64_t sk_iters;             // stream-K: tiles x kt_per_tile (0 = split-K grid)
  uint32_t kt_per_tile, tiles_n;
  uint32_t bk;                   // k-tile of the schedule (BK, or 32 with the TMA main loop)
  unsigned* status;              // watchdog word (TMA main loop waits)
  float* ws;                     // split-K [tiles][splits], stream-K [ctas][2]; 16 x 256 float4 each
  unsigned* counters;            // [tiles]
  uint32_t csk;                  // 1: the splits of a tile form one cluster (1, 1, splits) and
                                 //    reduce through distributed shared memory (TMA loop only)
};

// Global -> registers for one k-tile. A: thread -> row t/2, k (t%2)*BK/2 ...;
// B: thread -> k row t/(256/BK), columns (t%(256/BK))*BK/2 ...
template <bool VEC>
__device__ __forceinline__ void load_tile(const Params& p, uint32_t m0, uint32_t n0, uint32_t k0,
                                          uint32_t kend, float4 (&ra)[kLd], float4 (&rb)[kLdB]) {
  const uint32_t t = threadIdx.x;
  {
    const uint32_t r = m0 + t / 2;
    const bool rv = r < p.M;
    const float* a = p.A + size_t(r) * p.K;
#pragma unroll
    for (int q = 0; q < kLd; ++q) {
      const uint32_t k = k0 + (t % 2) * (BK / 2) + 4 * q;
      if (VEC) {
        ra[q] = (rv && k < kend) ? __ldg(reinterpret_cast<const float4*>(a + k))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        ra[q].x = (rv && k + 0 < kend) ? __ldg(a + k + 0) : 0.f;
        ra[q].y = (rv && k + 1 < kend) ? __ldg(a + k + 1) : 0.f;
        ra[q].z = (rv && k + 2 < kend) ? __ldg(a + k + 2) : 0.f;
        ra[q].w = (rv && k + 3 < kend) ? __ldg(a + k + 3) : 0.f;
      }
    }
  }
  {
    constexpr uint32_t tpr = 256 / BK;  // threads per B row
    const uint32_t k = k0 + t / tpr;
    const bool kv = k < kend;
    const float* b = p.B + size_t(k) * p.N;
#pragma unroll
    for (int q = 0; q < kLdB; ++q) {
      const uint32_t c = n0 + (t % tpr) * (4 * kLdB) + 4 * q;
      if (VEC) {
        rb[q] = (kv && c < p.N) ? __ldg(reinterpret_cast<const float4*>(b + c))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        rb[q].x = (kv && c + 0 < p.N) ? __ldg(b + c + 0) : 0.f;
        rb[q].y = (kv && c + 1 < p.N) ? __ldg(b + c + 1) : 0.f;
        rb[q].z = (kv && c + 2 < p.N) ? __ldg(b + c + 2) : 0.f;
        rb[q].w = (kv && c + 3 < p.N) ? __ldg(b + c + 3) : 0.f;
      }
    }
  }
}

__device__ __forceinline__ void store_tile(float (*As)[BM + APAD], float (*Bs)[BN],
                                           const float4 (&ra)[kLd], const float4 (&rb)[kLdB]) {
  const uint32_t t = threadIdx.x;
  const uint32_t r = t / 2;
#pragma unroll
  for (int q = 0; q < kLd; ++q) {
    const uint32_t k = (t % 2) * (BK / 2) + 4 * q;
    As[k + 0][r] = ra[q].x;
    As[k + 1][r] = ra[q].y;
    As[k + 2][r] = ra[q].z;
    As[k + 3][r] = ra[q].w;
  }
  constexpr uint32_t tpr = 256 / BK;
#pragma unroll
  for (int q = 0; q < kLdB; ++q)
    *reinterpret_cast<float4*>(&Bs[t / tpr][(t % tpr) * (4 * kLdB) + 4 * q]) = rb[q];
}

template <bool VEC>
__device__ __forceinline__ void store_out(const Params& p, uint32_t row, uint32_t col,
                                          const float (&v)[4]) {
  if (row >= p.M) return;
  float* c = p.C + size_t(row) * p.N + col;
  if (VEC && col + 3 < p.N) {
    float4 o = make_float4(p.alpha * v[0], p.alpha * v[1], p.alpha * v[2], p.alpha * v[3]);
    if (p.beta != 0.f) {
      const float4 old = *reinterpret_cast<const float4*>(c);
      o.x = fmaf(p.beta, old.x, o.x);
      o.y = fmaf(p.beta, old.y, o.y);
      o.z = fmaf(p.beta, old.z, o.z);
      o.w = fmaf(p.beta, old.w, o.w);
    }
    *reinterpret_cast<float4*>(c) = o;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (col + j < p.N) {
        float o = p.alpha * v[j];
        if (p.beta != 0.f) o = fmaf(p.beta, c[j], o);
        c[j] = o;
      }
    }
  }
}

// Partial 128 x 128 tile layout (float4 q of thread t at [q][t]: coalesced).
__device__ __forceinline__ void write_partial(float4* part, const float (&acc)[8][TN]) {
  const uint32_t t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int g = 0; g < NB; ++g)
      __stcg(part + (i * NB + g) * 256 + t,
             make_float4(acc[i][4 * g], acc[i][4 * g + 1], acc[i][4 * g + 2], acc[i][4 * g + 3]));
}

template <bool VEC>
__device__ __forceinline__ void store_acc(const Params& p, uint32_t m0, uint32_t n0,
                                          const float (&acc)[8][TN]) {
  const uint32_t t = threadIdx.x;
  const uint32_t tx = t % 16, ty = t / 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
#pragma unroll
    for (int g = 0; g < NB; ++g) {
      const float v[4] = {acc[i][4 * g], acc[i][4 * g + 1], acc[i][4 * g + 2], acc[i][4 * g + 3]};
      store_out<VEC>(p, row, n0 + 64 * g + tx * 4, v);
    }
  }
}

// acc = A[m0 : m0 + 128, kbeg : kend] * B[kbeg : kend, n0 : n0 + 128]. Ends with
// a barrier, so the shared-memory tiles may be reused right away.
template <bool VEC>
__device__ __forceinline__ void mainloop(const Params& p, uint32_t m0, uint32_t n0, uint32_t kbeg,
                                         uint32_t kend, float (*As)[BK][BM + APAD],
                                         float (*Bs)[BK][BN], float (&acc)[8][TN]) {
  const uint32_t t = threadIdx.x;
  const uint32_t tx = t % 16, ty = t / 16;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  const uint32_t nk = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
  float4 ra[kLd], rb[kLdB];
  if (nk > 0) {
    load_tile<VEC>(p, m0, n0, kbeg, kend, ra, rb);
    store_tile(As[0], Bs[0], ra, rb);
  }
  __syncthreads();

  for (uint32_t kt = 0; kt < nk; ++kt) {
    const uint32_t cur = kt & 1u;
    if (kt + 1 < nk) load_tile<VEC>(p, m0, n0, kbeg + (kt + 1) * BK, kend, ra, rb);
    // register double-buffered fragments: load step k+1 before the FFMAs of k
    float4 fa[2][2], fb[2][NB];
    fa[0][0] = *reinterpret_cast<const float4*>(&As[cur][0][ty * 4]);
    fa[0][1] = *reinterpret_cast<const float4*>(&As[cur][0][64 + ty * 4]);
#pragma unroll
    for (int g = 0; g < NB; ++g)
      fb[0][g] = *reinterpret_cast<const float4*>(&Bs[cur][0][64 * g + tx * 4]);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      const int c = k & 1, n = c ^ 1;
      if (k + 1 < BK) {
        fa[n][0] = *reinterpret_cast<const float4*>(&As[cur][k + 1][ty * 4]);
        fa[n][1] = *reinterpret_cast<const float4*>(&As[cur][k + 1][64 + ty * 4]);
#pragma unroll
        for (int g = 0; g < NB; ++g)
          fb[n][g] = *reinterpret_cast<const float4*>(&Bs[cur][k + 1][64 * g + tx * 4]);
      }
      const float a[8] = {fa[c][0].x, fa[c][0].y, fa[c][0].z, fa[c][0].w,
                          fa[c][1].x, fa[c][1].y, fa[c][1].z, fa[c][1].w};
      float b[TN];
#pragma unroll
      for (int g = 0; g < NB; ++g) {
        b[4 * g] = fb[c][g].x;
        b[4 * g + 1] = fb[c][g].y;
        b[4 * g + 2] = fb[c][g].z;
        b[4 * g + 3] = fb[c][g].w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) store_tile(As[cur ^ 1u], Bs[cur ^ 1u], ra, rb);
    __syncthreads();
  }
}

// ---------------------------------------------------------------- TMA main loop
// Used when A and B rows are 16-byte aligned (K % 4 == 0, N % 4 == 0). Per
// stage: the A tile [128 rows][32 k] and the B tile [32 k][128 n], fp32,
// unswizzled, loaded by TMA (zero fill past M, N, K). Thread 0 issues the
// loads; each warp releases a stage with one mbarrier arrival, so there is no
// CTA-wide barrier per k-tile and no register staging of global loads. A stays
// row-major: a thread reads its 8 rows as 8-byte (2 k) pieces.
constexpr int kTmaBk = 32;
constexpr int kTmaStages = 3;
// k values of A read per shared-memory load: 2 (LDS.64, 16 fragment
// registers). 4 (LDS.128) needs 16 more registers and spilled at the 128 that
// two CTAs per SM allow: 4096^3 45.4 vs 51.9 TFLOP/s.
constexpr int kTmaAk = 2;
// the one-CTA-per-SM loop (4-k A reads) has the registers to unroll four
// groups: 1024^3 65.5 -> 61.5-62.0 us (2: 62.5, 8: 63.0-63.5)
constexpr int kAk4Unroll = 4;
// A tile of AP floats per row (AP = row pitch). AP = 32: the rows a warp reads
// at once (4 apart) share banks, a 2-way conflict on every A load. AP = 36: the
// box is 36 k wide (the last 4 columns are the next k-tile's, unused) and the
// 144-byte pitch puts those rows in different banks; each row then spans two
// L2 lines. Measured: 36 is faster for K <= 2048 (1024^3 69.6 -> 67.6 us,
// 2048^3 390 -> 376 us), 32 for long K (4096^3 2650 vs 2803 us).
// The k-tile follows from the pitch: AP = 32 / 36 take 32-deep k-tiles, AP =
// 64 / 68 (the same two layouts) 64-deep ones. The cluster split-K kernel (one
// CTA per SM, room for 3 x 67.6 KB of stages) takes the 64-deep tiles: half
// the barrier waits and loop trips per FFMA (1024^3 61.4 -> 59.4 us,
// 300 x 520 x 2004 36.9 -> 34.8 us).
template <int AP>
struct TmaTile {
  static constexpr int kBk = AP & ~31;
  static_assert(kBk == 32 || kBk == 64, "A row pitch");
  static constexpr int kA = BM * AP * 4;
  static constexpr int kB = kBk * BN * 4;
  static constexpr int kSmem = kTmaStages * (kA + kB) + 2 * kTmaStages * 8 + 16;
};
static_assert(BN == 128, "TMA main loop: 128 x 128 tiles");

struct TmaPipe {
  uint32_t tr_seg;  // trace builds: segment index of the current main loop
  float* sA;
  float* sB;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;
  uint32_t kt_load, kt_use;  // k-tiles issued / consumed by this CTA so far
};

template <int AP>
__device__ __forceinline__ bool tma_issue(TmaPipe& q, const CUtensorMap* tmA,
                                          const CUtensorMap* tmB, const Params& p, uint32_t m0,
                                          uint32_t n0, uint32_t kb) {
  const uint32_t st = q.kt_load % kTmaStages, use = q.kt_load / kTmaStages;
  if (!felix_sm100::mbar_wait(q.empty + st, (use & 1u) ^ 1u, q.abort_flag, p.status,
                              felix_sm100::kWdProducerEmpty))
    return false;
  constexpr int kBk = TmaTile<AP>::kBk;
  felix_sm100::mbar_arrive_expect_tx(q.full + st, TmaTile<AP>::kA + TmaTile<AP>::kB);
  felix_sm100::tma_load_2d(q.sA + st * (TmaTile<AP>::kA / 4), tmA, q.full + st, int(kb * kBk),
                           int(m0));
  felix_sm100::tma_load_2d(q.sB + st * (TmaTile<AP>::kB / 4), tmB, q.full + st, int(n0),
                           int(kb * kBk));
  ++q.kt_load;
  return true;
}

// acc = A[m0 : m0 + 128, kbeg : kend] * B[kbeg : kend, n0 : n0 + 128] with
// kbeg a multiple of 32 (k past kend inside the last k-tile must be past K).
template <int AP, int AK = kTmaAk>
__device__ __forceinline__ bool mainloop_tma(TmaPipe& q, const CUtensorMap* tmA,
                                             const CUtensorMap* tmB, const Params& p,
                                             uint32_t m0, uint32_t n0, uint32_t kbeg,
                                             uint32_t kend, float (&acc)[8][TN]) {
  const uint32_t t = threadIdx.x, lane = t % 32;
  const uint32_t tx = t % 16, ty = t / 16;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  constexpr int kBk = TmaTile<AP>::kBk;
  const uint32_t kb0 = kbeg / kBk;
  const uint32_t n = kend > kbeg ? (kend - kbeg + kBk - 1) / kBk : 0;
  bool ok = true;
  if (t == 0)
    for (uint32_t j = 0; ok && j < n && j < kTmaStages - 1; ++j)
      ok = tma_issue<AP>(q, tmA, tmB, p, m0, n0, kb0 + j);
  for (uint32_t j = 0; j < n; ++j) {
    const uint32_t st = q.kt_use % kTmaStages;
    if (!felix_sm100::mbar_wait(q.full + st, (q.kt_use / kTmaStages) & 1u, q.abort_flag, p.status,
                                felix_sm100::kWdMmaFull))
      return false;
    if (j == 0) SG_TR(q.tr_seg * 3 + 1);
    const float* a_s = q.sA + st * (TmaTile<AP>::kA / 4);  // [128][AP]
    const float* b_s = q.sB + st * (TmaTile<AP>::kB / 4);  // [kBk][128]
    // one group of AK k-steps per iteration; the 2-k loop is not unrolled:
    // unrolled, the compiler hoists the B loads of later groups and spills at
    // 128 registers
#pragma unroll(AK == 4 ? kAk4Unroll : 1)
    for (int k2 = 0; k2 < kBk / AK; ++k2) {
      // A: AK consecutive k of each of the thread's 8 rows per load
      float af[8][AK];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t row = i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4);
        if constexpr (AK == 4) {
          const float4 v = *reinterpret_cast<const float4*>(a_s + row * AP + k2 * AK);
          af[i][0] = v.x;
          af[i][1] = v.y;
          af[i][2 % AK] = v.z;
          af[i][3 % AK] = v.w;
        } else {
          const float2 v = *reinterpret_cast<const float2*>(a_s + row * AP + k2 * AK);
          af[i][0] = v.x;
          af[i][1] = v.y;
        }
      }
#pragma unroll
      for (int kk = 0; kk < AK; ++kk) {
        const int k = k2 * AK + kk;
        float b[TN];
#pragma unroll
        for (int g = 0; g < NB; ++g) {
          const float4 bv = *reinterpret_cast<const float4*>(b_s + k * BN + 64 * g + tx * 4);
          b[4 * g] = bv.x;
          b[4 * g + 1] = bv.y;
          b[4 * g + 2] = bv.z;
          b[4 * g + 3] = bv.w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int jj = 0; jj < TN; ++jj) acc[i][jj] = fmaf(af[i][kk], b[jj], acc[i][jj]);
      }
    }
    __syncwarp();
    if (lane == 0) felix_sm100::mbar_arrive(q.empty + st);
    ++q.kt_use;
    if (t == 0 && ok && j + kTmaStages - 1 < n)
      ok = tma_issue<AP>(q, tmA, tmB, p, m0, n0, kb0 + j + kTmaStages - 1);
  }
  return true;
}

// Before the CTA exits: every TMA load it issued has landed (a load can still
// be in flight only after an aborted wait).
template <bool TMA>
__device__ __forceinline__ void drain_tma(TmaPipe& q, const Params& p) {
  if constexpr (TMA) {
    if (threadIdx.x == 0) {
      int dummy = 0;
      for (uint32_t k = q.kt_use; k < q.kt_load; ++k)
        felix_sm100::mbar_wait(q.full + k % kTmaStages, (k / kTmaStages) & 1u, &dummy, p.status,
                               felix_sm100::kWdDrain, 100000000ull);
    }
  }
}

// Cluster split-K reduction: CTA `rank` of the (1, 1, S) cluster sums rows
// [rank * 128 / S, (rank + 1) * 128 / S) of the S partial tiles parked at
// red_addr in every CTA of the cluster, in rank order (deterministic), and
// writes them to C. All S x U loads of a thread are issued before the first
// sum, so the distributed-shared-memory latency is paid once, not per row.
template <bool VEC, uint32_t S>
__device__ __forceinline__ void csk_reduce(const Params& p, uint32_t m0, uint32_t n0,
                                           uint32_t rank, uint32_t red_addr, bool ok) {
  constexpr uint32_t kRows = BM / S, kF4 = kRows * (BN / 4), U = kF4 / kThreads;
  static_assert(kF4 % kThreads == 0, "cluster reduction: whole float4s per thread");
  const uint32_t t = threadIdx.x;
  float4 x[U][S];
#pragma unroll
  for (uint32_t u = 0; u < U; ++u) {
    const uint32_t f = t + u * kThreads;
    const uint32_t off = ((rank * kRows + f / (BN / 4)) * BN + (f % (BN / 4)) * 4) * 4;
#pragma unroll
    for (uint32_t src = 0; src < S; ++src)
      x[u][src] = felix_sm100::ld_shared_cluster_v4f(felix_sm100::mapa_shared(red_addr + off, src));
  }
#pragma unroll
  for (uint32_t u = 0; u < U; ++u) {
    const uint32_t f = t + u * kThreads;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (uint32_t src = 0; src < S; ++src) {
      sum.x += x[u][src].x;
      sum.y += x[u][src].y;
      sum.z += x[u][src].z;
      sum.w += x[u][src].w;
    }
    const float v[4] = {sum.x, sum.y, sum.z, sum.w};
    if (ok) store_out<VEC>(p, m0 + rank * kRows + f / (BN / 4), n0 + (f % (BN / 4)) * 4, v);
  }
}

// Stream-K: CTA of iteration x (iterations = tiles x k-tiles, split evenly).
__device__ __forceinline__ uint32_t sk_cta_of(uint64_t x, uint32_t P, uint64_t I) {
  return static_cast<uint32_t>(((x + 1) * P - 1) / I);
}

// CSK: the cluster split-K instantiation, one CTA per SM (up to 255
// registers), so its main loop reads A 4 k at a time (128-bit loads); the
// plain kernels keep two CTAs per SM at 128 registers and 2-k A reads.
template <bool VEC, bool TMA, int AP = 32, bool CSK = false>
__global__ void __launch_bounds__(kThreads, CSK ? 1 : FELIX_SGEMM_MINB)
    sgemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const Params p) {
  extern __shared__ __align__(1024) uint8_t dsmem[];
  __shared__ uint32_t s_last;
  __shared__ int s_abort;
  const uint32_t t = threadIdx.x;
  float acc[8][TN];
  // register-staged main loop: As [2][BK][BM + APAD], Bs [2][BK][BN]
  auto As = reinterpret_cast<float(*)[BK][BM + APAD]>(dsmem);
  auto Bs = reinterpret_cast<float(*)[BK][BN]>(dsmem + 2 * BK * (BM + APAD) * 4);
  // TMA main loop: stages of A and B tiles, then the full / empty barriers
  TmaPipe q{};
  if constexpr (TMA) {
    q.sA = reinterpret_cast<float*>(dsmem);
    q.sB = reinterpret_cast<float*>(dsmem + kTmaStages * TmaTile<AP>::kA);
    q.full = reinterpret_cast<uint64_t*>(dsmem + kTmaStages * (TmaTile<AP>::kA + TmaTile<AP>::kB));
    q.empty = q.full + kTmaStages;
    q.abort_flag = &s_abort;
    if (t == 0) {
      for (int i = 0; i < kTmaStages; ++i) {
        felix_sm100::mbar_init(q.full + i, 1);
        felix_sm100::mbar_init(q.empty + i, kThreads / 32);
      }
      s_abort = 0;
      felix_sm100::fence_mbar_init();
      felix_sm100::tma_prefetch_desc(&tmA);
      felix_sm100::tma_prefetch_desc(&tmB);
    }
    __syncthreads();
  }
  SG_TR(0);
  auto run = [&](uint32_t m0, uint32_t n0, uint32_t kbeg, uint32_t kend) -> bool {
    if constexpr (TMA) {
      return mainloop_tma<AP, CSK ? 4 : kTmaAk>(q, &tmA, &tmB, p, m0, n0, kbeg, kend, acc);
    } else {
      mainloop<VEC>(p, m0, n0, kbeg, kend, As, Bs, acc);
      return true;
    }
  };

  if (p.sk_iters != 0) {
    // ------------------------------------------------------------ stream-K
    // CTA c owns iterations [I c / P, I (c + 1) / P) of the (tile, k-tile)
    // sequence; a tile it covers only in part goes to one of its two partial
    // slots, and the last of the tile's CTAs to finish sums the slots in CTA
    // order (deterministic) and writes C.
    const uint32_t P = gridDim.x, c = blockIdx.x;
    const uint64_t I = p.sk_iters;
    const uint32_t KT = p.kt_per_tile;
    const uint64_t start = I * c / P, end = I * (c + 1) / P;
    uint64_t it = start;
    while (it < end) {
      const uint32_t tile = static_cast<uint32_t>(it / KT);
      const uint32_t kb0 = static_cast<uint32_t>(it - uint64_t(tile) * KT);
      const uint64_t left = end - it;
      const uint32_t kb1 = left < uint64_t(KT - kb0) ? kb0 + static_cast<uint32_t>(left) : KT;
      const uint32_t m0 = (tile / p.tiles_n) * BM, n0 = (tile % p.tiles_n) * BN;
      q.tr_seg = it == start ? 0u : 1u;
      if (!run(m0, n0, kb0 * p.bk, min(p.K, kb1 * p.bk))) break;
      SG_TR(q.tr_seg * 3 + 2);
      if (kb0 == 0 && kb1 == KT) {
        store_acc<VEC>(p, m0, n0, acc);
      } else {
        const uint32_t seg = it == start ? 0u : 1u;
        write_partial(reinterpret_cast<float4*>(p.ws) + (size_t(c) * 2 + seg) * (kPartF4 * 256),
                      acc);
        __threadfence();
        __syncthreads();
        const uint32_t c_first = sk_cta_of(uint64_t(tile) * KT, P, I);
        const uint32_t c_last = sk_cta_of(uint64_t(tile + 1) * KT - 1, P, I);
        if (t == 0) {
          const unsigned old = atomicAdd(&p.counters[tile], 1u);
          const uint32_t last = old == c_last - c_first ? 1u : 0u;
          if (last) atomicExch(&p.counters[tile], 0u);
          s_last = last;
        }
        __syncthreads();
        if (s_last) {
          __threadfence();
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
          for (uint32_t cc = c_first; cc <= c_last; ++cc) {
            // the tile is CTA cc's first segment when cc starts inside it
            const uint32_t sg = I * cc / P >= uint64_t(tile) * KT ? 0u : 1u;
            const float4* part =
                reinterpret_cast<const float4*>(p.ws) + (size_t(cc) * 2 + sg) * (kPartF4 * 256);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
              for (int g = 0; g < NB; ++g) {
                const float4 x = __ldcg(part + (i * NB + g) * 256 + t);
                acc[i][4 * g] += x.x;
                acc[i][4 * g + 1] += x.y;
                acc[i][4 * g + 2] += x.z;
                acc[i][4 * g + 3] += x.w;
              }
          }
          store_acc<VEC>(p, m0, n0, acc);
        }
      }
      SG_TR(q.tr_seg * 3 + 3);
      it += kb1 - kb0;
    }
    drain_tma<TMA>(q, p);
    SG_TR(7);
    return;
  }

  // -------------------------------------------------------------- split-K
  const uint32_t m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const uint32_t z = blockIdx.z;
  const uint32_t kbeg = z * p.k_per_split;
  const uint32_t kend = min(p.K, kbeg + p.k_per_split);
  const bool ok = run(m0, n0, kbeg, kend);
  SG_TR(2);
  drain_tma<TMA>(q, p);
  // (a separate instantiation: the cluster epilogue in the same kernel as the
  // plain one changed the main loop's code and cost 16 % at 4096^3)
  if constexpr (TMA && CSK) {
    {
      // Cluster split-K: each CTA parks its fp32 partial tile in its own
      // (now idle) TMA ring, then CTA r of the cluster sums rows
      // [r * 128 / S, (r + 1) * 128 / S) of all S partials in rank order
      // (deterministic) over distributed shared memory and writes C. Every
      // CTA reaches both cluster barriers, also after an aborted wait.
      float* red = reinterpret_cast<float*>(dsmem);  // [128][128]
      __syncthreads();  // every warp is done with the ring
      if (ok) {
        const uint32_t tx = t % 16, ty = t / 16;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t row = i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4);
#pragma unroll
          for (int g = 0; g < NB; ++g)
            *reinterpret_cast<float4*>(red + row * BN + 64 * g + tx * 4) =
                make_float4(acc[i][4 * g], acc[i][4 * g + 1], acc[i][4 * g + 2],
                            acc[i][4 * g + 3]);
        }
      }
      felix_sm100::cluster_sync();
      const uint32_t red_addr = felix_sm100::smem_u32(red);
      SG_TR(3);
      if (gridDim.z == 2)
        csk_reduce<VEC, 2>(p, m0, n0, z, red_addr, ok);
      else if (gridDim.z == 4)
        csk_reduce<VEC, 4>(p, m0, n0, z, red_addr, ok);
      else
        csk_reduce<VEC, 8>(p, m0, n0, z, red_addr, ok);
      SG_TR(4);
      felix_sm100::cluster_sync();  // no CTA exits while another reads its ring
      return;
    }
  }
  if (!ok) return;

  if (p.splits == 1) {
    store_acc<VEC>(p, m0, n0, acc);
    return;
  }

  // Split-K: publish the partial; the last split of the tile to finish sums
  // the partials in split order.
  const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
  write_partial(reinterpret_cast<float4*>(p.ws) + (size_t(tile) * p.splits + z) * (kPartF4 * 256),
                acc);
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const unsigned old = atomicAdd(&p.counters[tile], 1u);
    const uint32_t last = old == p.splits - 1 ? 1u : 0u;
    if (last) atomicExch(&p.counters[tile], 0u);
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float4* base =
      reinterpret_cast<const float4*>(p.ws) + size_t(tile) * p.splits * (kPartF4 * 256);
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int g = 0; g < NB; ++g) {
      float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (uint32_t zz = 0; zz < p.splits; ++zz) {
        const float4 x0 = __ldcg(base + zz * (kPartF4 * 256) + (i * NB + g) * 256 + t);
        s0.x += x0.x; s0.y += x0.y; s0.z += x0.z; s0.w += x0.w;
      }
      acc[i][4 * g] = s0.x;
      acc[i][4 * g + 1] = s0.y;
      acc[i][4 * g + 2] = s0.z;
      acc[i][4 * g + 3] = s0.w;
    }
  store_acc<VEC>(p, m0, n0, acc);
}

}  // namespace sgemm
}  // namespace felix_sm100

#ifdef FELIX_SGEMM_TRACE
extern "C" void sg_trace_fetch(void* dst) {
  cudaMemcpyFromSymbol(dst, felix_sm100::sgemm::g_sg_trace, sizeof(felix_sm100::sgemm::g_sg_trace));
}
#endif

// Scratch of felix_sgemm_noalloc: the fixed counter block followed by room
// for 256 partial 128 x 128 fp32 tiles (16 MiB + 16 KiB). It is part of the
// library's device image, so every GPU that loads the library holds it until
// the process exits. Zero-initialised at load; the kernel leaves the counters
// at zero and the entry point clears them again before every launch.
constexpr size_t kNoAllocPartialBytes = size_t(16) << 20;
constexpr size_t kNoAllocScratchBytes = felix_impl::kWsCounterBytes + kNoAllocPartialBytes;
static __device__ __align__(256) unsigned char g_sgemm_noalloc_scratch[kNoAllocScratchBytes];

namespace felix_impl {

using namespace felix_sm100::sgemm;

namespace {
uint32_t choose_splits(uint32_t M, uint32_t N, uint32_t K, const SgemmOptions& o, int num_sms) {
  const uint32_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  uint32_t s;
  if (o.split_k > 0) {
    s = uint32_t(o.split_k);
  } else {
    // Aim for two resident CTAs per SM, keeping at least 128 of K per split.
    const uint32_t target = 2u * uint32_t(num_sms);
    s = tiles >= target ? 1u : target / tiles;
    const uint32_t kmax = K / 128u;
    if (s > kmax) s = kmax;
    if (s < 1) s = 1;
    if (s > 16) s = 16;
  }
  const uint32_t kblocks = (K + BK - 1) / BK;
  if (s > kblocks) s = kblocks ? kblocks : 1;
  if (tiles > kWsMaxCounters) s = 1;  // one counter per tile lives in the fixed block
  return s;
}
}  // namespace

// Stream-K grid (0 = use the split-K grid): when the 128 x 128 tiles do not
// fill one wave of two resident CTAs per SM, spread (tile, k-tile)
// iterations evenly over 2 x SMs CTAs (each at least 4 k-tiles).
uint32_t choose_stream_k(uint32_t M, uint32_t N, uint32_t K, const SgemmOptions& o, int num_sms,
                         uint32_t bk) {
  if (o.split_k != 0 || !o.allow_stream_k) return 0;
  const uint32_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const uint32_t kt = (K + bk - 1) / bk;
  const uint32_t slots = uint32_t(FELIX_SGEMM_MINB) * uint32_t(num_sms);
  // (with a full wave or more, plain tiles measured as fast: 4096^3 43.9 vs
  // 43.3 TFLOP/s)
  if (kt < 8 || tiles >= slots || tiles > kWsMaxCounters) return 0;
  const uint64_t iters = uint64_t(tiles) * kt;
  uint64_t P = slots;
  if (P > iters / 4) P = iters / 4;
  return P >= 2 ? uint32_t(P) : 0;
}

size_t sgemm_workspace_bytes(uint32_t M, uint32_t N, uint32_t K, const SgemmOptions& o,
                             int num_sms) {
  // (the larger of the two main loops' needs: the k-tile is BK or 32)
  const uint32_t P = choose_stream_k(M, N, K, o, num_sms, BK);
  if (P) return kWsCounterBytes + size_t(P) * 2 * BM * BN * sizeof(float);
  const uint32_t s = choose_splits(M, N, K, o, num_sms);
  if (s <= 1) return 0;
  const size_t tiles = size_t((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  return kWsCounterBytes + tiles * s * BM * BN * sizeof(float);
}

FelixCode sgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                       const float* B, float beta, float* C, const SgemmOptions& o,
                       void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (M == 0 || N == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  if (!C || (K > 0 && (!A || !B))) return api_error("sgemm: null pointer");
  if (K == 0) return scale_float_matrix(C, size_t(M) * N, beta, stream);
  DeviceInfo* dev = current_device_info();
  if (!dev) return launch_error(cudaGetLastError(), "sgemm: no CUDA device");

  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.A = A;
  p.B = B;
  p.C = C;
  const bool vec = (K % 4 == 0) && (N % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
                     reinterpret_cast<uintptr_t>(C)) &
                    15u) == 0;
  // TMA main loop: rows of A and B must be 16-byte multiples (vec)
  const bool tma = vec && o.allow_tma;
  p.bk = tma ? uint32_t(kTmaBk) : uint32_t(BK);
  p.status = dev->status_word;
  CUtensorMap tmA{}, tmB{};
  const int ap = K <= 2048 ? 36 : 32;  // A row pitch (TmaTile)
  if (tma) {
    if (encode_tmap_2d_f32(&tmA, A, K, M, uint64_t(K) * 4, uint32_t(ap), BM) ||
        encode_tmap_2d_f32(&tmB, B, N, K, uint64_t(N) * 4, BN, kTmaBk))
      return api_error("sgemm: cuTensorMapEncodeTiled failed");
    static PerDeviceOnce once;
    const int rc = once.run(dev->ordinal, [] {
      cudaError_t e = cudaFuncSetAttribute(sgemm_kernel<true, true, 32>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           TmaTile<32>::kSmem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(sgemm_kernel<true, true, 36>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, TmaTile<36>::kSmem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(sgemm_kernel<true, true, 64, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, TmaTile<64>::kSmem);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(sgemm_kernel<true, true, 68, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, TmaTile<68>::kSmem);
      return int(e);
    });
    if (rc < 0) return api_error("sgemm: device ordinal");
    if (rc > 0) return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
  }
  auto launch = [&](dim3 grid) -> FelixCode {
    constexpr size_t kRegSmem = size_t(2) * BK * (BM + APAD) * 4 + size_t(2) * BK * BN * 4;
    if (tma && ap == 36)
      sgemm_kernel<true, true, 36><<<grid, kThreads, TmaTile<36>::kSmem, stream>>>(tmA, tmB, p);
    else if (tma)
      sgemm_kernel<true, true, 32><<<grid, kThreads, TmaTile<32>::kSmem, stream>>>(tmA, tmB, p);
    else if (vec)
      sgemm_kernel<true, false><<<grid, kThreads, kRegSmem, stream>>>(tmA, tmB, p);
    else
      sgemm_kernel<false, false><<<grid, kThreads, kRegSmem, stream>>>(tmA, tmB, p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return launch_error(e, "sgemm: launch failed");
    return FelixCode{FELIX_SUCCESS, cudaSuccess};
  };
  auto attach = [&](size_t need) -> FelixCode {
    if (!workspace) {
      if (o.forbid_alloc) return api_error("sgemm: split-K scratch missing on an allocation-free call");
      workspace = library_workspace(dev, stream, need);
      if (!workspace) return launch_error(cudaErrorMemoryAllocation, "sgemm: workspace");
    } else if (ws_bytes < need) {
      return api_error("sgemm: workspace too small");
    }
    p.counters = static_cast<unsigned*>(workspace);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsCounterBytes);
    return FelixCode{FELIX_SUCCESS, cudaSuccess};
  };

  // Cluster split-K (TMA loop): tiles well short of one wave of two CTAs per
  // SM get S = 2, 4 or 8 K-splits per tile as one (1, 1, S) cluster that
  // reduces on chip, instead of stream-K partials in global memory, while
  // each split stays short (<= 16 k-tiles; longer K balances better with
  // stream-K). Measured (us, cluster vs stream-K, timing loop): 1024^3 65.5 vs 69.6,
  // 1000^3 65.5 vs 69.7, 300 x 520 x 2004 41.0 vs 65.5; 2048 x 1024 x 4096
  // 459 vs 401 and 512 x 512 x 8192 236 vs 127 (left to stream-K).
  {
    const uint32_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const uint32_t slots = uint32_t(dev->num_sms);  // one cluster-split CTA per SM
    const uint32_t kt = (K + p.bk - 1) / p.bk;
    uint32_t S = 0;
    if (tma && o.split_k == 0 && o.allow_stream_k && tiles * 2 <= slots) {
      S = slots / tiles >= 8 ? 8u : slots / tiles >= 4 ? 4u : 2u;
      while (S > 1 && kt < 4 * S) S /= 2;
      if (S >= 2 && (kt + S - 1) / S > 16) S = 0;
    }
    if (S >= 2 && (M + BM - 1) / BM <= 65535u) {
      // 64-deep k-tiles: their own tensor maps (A box 68 or 64 wide, B box 64 high)
      const int ap64 = ap + 32;
      CUtensorMap tmA64{}, tmB64{};
      if (encode_tmap_2d_f32(&tmA64, A, K, M, uint64_t(K) * 4, uint32_t(ap64), BM) ||
          encode_tmap_2d_f32(&tmB64, B, N, K, uint64_t(N) * 4, BN, 64))
        return api_error("sgemm: cuTensorMapEncodeTiled failed");
      p.bk = 64;
      const uint32_t kt64 = (K + 63) / 64;
      p.csk = 1;
      p.splits = S;
      p.k_per_split = ((kt64 + S - 1) / S) * 64;
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3((N + BN - 1) / BN, (M + BM - 1) / BM, S);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = ap64 == 68 ? TmaTile<68>::kSmem : TmaTile<64>::kSmem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = S;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      const cudaError_t e =
          ap64 == 68 ? cudaLaunchKernelEx(&cfg, sgemm_kernel<true, true, 68, true>, tmA64, tmB64, p)
                     : cudaLaunchKernelEx(&cfg, sgemm_kernel<true, true, 64, true>, tmA64, tmB64, p);
      if (e != cudaSuccess) return launch_error(e, "sgemm: cluster launch failed");
      return FelixCode{FELIX_SUCCESS, cudaSuccess};
    }
  }
  const uint32_t sk_ctas = choose_stream_k(M, N, K, o, dev->num_sms, p.bk);
  if (sk_ctas) {
    p.tiles_n = (N + BN - 1) / BN;
    p.kt_per_tile = (K + p.bk - 1) / p.bk;
    p.sk_iters = uint64_t(p.tiles_n) * ((M + BM - 1) / BM) * p.kt_per_tile;
    p.splits = 1;
    FelixCode rc = attach(kWsCounterBytes + size_t(sk_ctas) * 2 * BM * BN * sizeof(float));
    if (rc.type != FELIX_SUCCESS) return rc;
    return launch(dim3(sk_ctas));
  }
  p.splits = choose_splits(M, N, K, o, dev->num_sms);
  const uint32_t kblocks = (K + p.bk - 1) / p.bk;
  if (p.splits > kblocks) p.splits = kblocks;
  p.k_per_split = ((kblocks + p.splits - 1) / p.splits) * p.bk;
  // Recompute the split count so that no split is empty.
  p.splits = (K + p.k_per_split - 1) / p.k_per_split;
  const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, p.splits);
  if (grid.y > 65535u) return api_error("sgemm: M too large");
  if (p.splits > 1) {
    const size_t tiles = size_t(grid.x) * grid.y;
    FelixCode rc = attach(kWsCounterBytes + tiles * p.splits * BM * BN * sizeof(float));
    if (rc.type != FELIX_SUCCESS) return rc;
  }
  return launch(grid);
}

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};
}  // namespace

// Device address of the static scratch on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device, with that device current, and cached.
static void* noalloc_scratch(int device, cudaError_t* err) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_sgemm_noalloc_scratch);
    if (e != cudaSuccess) {
      *err = e;
      return nullptr;
    }
    g_noalloc_ptr[device] = ptr;
  }
  return g_noalloc_ptr[device];
}

FelixCode sgemm_noalloc_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                               const float* B, float beta, float* C, int split_k,
                               cudaStream_t stream) {
  if (split_k < 0) return api_error("sgemm_noalloc: split_k must be >= 0");
  if (M == 0 || N == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  if (K == 0) return sgemm_launch(M, N, K, alpha, A, B, beta, C, SgemmOptions{}, nullptr, 0, stream);
  DeviceInfo* dev = current_device_info();
  if (!dev) return launch_error(cudaGetLastError(), "sgemm_noalloc: no CUDA device");
  SgemmOptions o;
  o.split_k = split_k;
  o.allow_stream_k = false;  // the static scratch is sized for split-K partials
  o.allow_tma = false;
  o.forbid_alloc = true;     // a mismatch below becomes an error, never a cudaMalloc
  const uint32_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  constexpr uint32_t kMaxPartials = uint32_t(kNoAllocPartialBytes / (size_t(BM) * BN * sizeof(float)));
  // The limit is checked on the split the caller asked for, before any clamping.
  if (split_k > 1 && uint64_t(tiles) * uint64_t(split_k) > kMaxPartials)
    return api_error(
        "sgemm_noalloc: this split_k needs more split-K scratch than the 16 MiB static "
        "scratch holds (at most 256 partial 128x128 tiles: tiles x split_k <= 256)");
  size_t need = sgemm_workspace_bytes(M, N, K, o, dev->num_sms);
  if (need > kNoAllocScratchBytes) {
    // automatic split: the largest one whose partial tiles fit
    o.split_k = int(kMaxPartials / tiles);
    if (o.split_k < 1) o.split_k = 1;
    need = sgemm_workspace_bytes(M, N, K, o, dev->num_sms);
  }
  if (need > kNoAllocScratchBytes) return api_error("sgemm_noalloc: scratch size mismatch");
  void* scratch = nullptr;
  if (need > 0) {
    cudaError_t e = cudaSuccess;
    scratch = noalloc_scratch(dev->ordinal, &e);
    if (!scratch) return launch_error(e, "sgemm_noalloc: cudaGetSymbolAddress(scratch)");
    // the tile counters must start at zero
    e = cudaMemsetAsync(scratch, 0, kWsCounterBytes, stream);
    if (e != cudaSuccess) return launch_error(e, "sgemm_noalloc: clearing the counters");
  }
  return sgemm_launch(M, N, K, alpha, A, B, beta, C, o, scratch, kNoAllocScratchBytes, stream);
}

}  // namespace felix_impl
