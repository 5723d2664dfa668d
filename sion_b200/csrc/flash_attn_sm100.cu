// Flash-attention forward for sm_100a, fp16 in/out, no mask:
//   O = softmax(Q K^T * scale) V per (batch, head), plus the fp32 natural-log
//   log-sum-exp of every query row.
// Replaces the Ampere mma.sync kernel behind felix::ampere_flash_attn_launch
// (reference: src/felix/flash_attention/ampere_flash_attn_mma16168_64_1D_warp_tiling_kernel_launch.cu:8-55,
// kernels/ampere_flash_attn_mma16168_64_1D_warp_tiling.cuh:23-466), which keeps S
// and O in fp16, fixes scale = 1/sqrt(D), requires seqlen % 64 == 0 and has no
// LSE output. Here S and O accumulate in fp32 (TMEM), any seqlen >= 1 works
// (TMA zero-fills the ragged tail, the softmax masks it), and LSE is written.
//
// Layout: Q, K, V, O are [B, H, S, D] contiguous; LSE is [B, H, S].
//
// Work item = one (b, h) and 256 query rows as two 128-row tiles "A" and "B";
// a CTA takes one item, or (persistent launch, non-causal) strides over items.
//   warp 0      TMA loader: Q_A, Q_B once, then the K ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warp 2      TMA loader of the V ring
//   warps 4-7   softmax of tile A (one query row per thread)
//   warps 8-11  softmax of tile B
// TMEM (512 columns): S_A | S_B | O_A | O_B, 128 columns each (D = 128);
// P (fp16, two per 32-bit column) overwrites the first half of its S tile.
// Per KV block j the issue order is PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), so
// the softmax of one tile overlaps the tensor-core work of the other. S_t(j+1)
// is issued right behind PV_t(j): the tensor pipe executes a CTA's MMAs in
// issue order, so S_t(j+1)'s writes cannot overtake PV_t(j)'s reads of P_t.
// K and V have separate rings so K(j+1) streams in while V(j) is still used.
// Online softmax in the log2 domain with packed fp32x2 arithmetic; O and l are
// rescaled only when the row maximum grows by more than 8 (P then stays below
// 2^8, safe in fp16), and O is normalised once at the end.
#include <cstdio>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "felix_internal.h"
#include "sm100_ptx.cuh"

namespace felix_sm100 {
namespace attn {

constexpr int kBlockQ = 128;   // rows per Q tile (UMMA M)
constexpr int kBlockKV = 128;  // keys per KV block (UMMA N of QK^T, K of PV)
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Register split: the kernel launches with 168 registers per thread (384
// threads); warpgroup 0 (loaders, MMA issuer; it spills below 80) drops to 80
// and the two softmax warpgroups rise to 200, so a softmax thread holds its
// whole 128-column S row (loaded with one wait) without spilling.
// setmaxnreg.inc draws on the registers the block was launched with:
// 80 x 128 + 200 x 256 = 61440 <= 168 x 384 = 64512. The host refuses to
// launch if the compiled kernel's count differs from 168.
#ifndef FELIX_FA_REGSPLIT
#define FELIX_FA_REGSPLIT 1
#endif
constexpr bool kRegSplit = FELIX_FA_REGSPLIT != 0;
constexpr int kRegsLaunch = 168, kRegsSide = 80, kRegsSoftmax = 200;
static_assert(kRegsSide * 128 + kRegsSoftmax * 256 <= kRegsLaunch * kThreads, "register split");

// CG = 1: one CTA per 256 query rows. CG = 2 (D = 128): a cluster of two CTAs
// per 512 query rows whose MMAs are cta_group::2 (M = 256); each CTA then
// holds half of every K block (64 keys) and half of every V block (64 of the
// D columns), so per-SM shared-memory operand traffic drops by ~40%.
template <int D, int CG>
struct Cfg {
#ifdef FELIX_FA_KST
  static constexpr int kKStages = FELIX_FA_KST;
  static constexpr int kVStages = FELIX_FA_VST;
#else
  static constexpr int kKStages = CG == 2 ? 4 : (D == 128 ? 3 : 4);  // K ring
  static constexpr int kVStages = CG == 2 ? 4 : (D == 128 ? 2 : 4);  // V ring
#endif
  static constexpr int kChunks = D / 64;                 // 128-byte swizzle chunks per row
  static constexpr int kTileBytes = kBlockQ * D * 2;     // one 128 x D fp16 Q tile
  static constexpr int kKeys = kBlockKV / CG;            // K rows held per CTA
  static constexpr int kKBytes = kKeys * D * 2;          // K slot
  static constexpr int kVCols = D / CG;                  // V columns held per CTA
  static constexpr int kVBytes = kBlockKV * kVCols * 2;  // V slot
  static constexpr int kQOff = 0;                        // Q_A, Q_B
  static constexpr int kKOff = 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kKStages * kKBytes;
  static constexpr int kBarOff = kVOff + kVStages * kVBytes;
  static constexpr int kSmemBytes = kBarOff + 256 + 1024;
  static_assert(CG == 1 || D == 128, "CTA pairs need D = 128");
};

// TMEM columns of tile t's S (and P) and O accumulators.
__device__ __forceinline__ uint32_t col_s(int t) { return uint32_t(t) * 128u; }
__device__ __forceinline__ uint32_t col_o(int t) { return 256u + uint32_t(t) * 128u; }

struct Params {
  __half* O;
  float* lse;
  uint32_t S;        // sequence length
  uint32_t n_kv;     // KV blocks
  uint32_t q_tiles;  // CTA groups per (b, h) along the query axis
  float scale_log2;  // scale * log2(e)
  uint32_t causal;   // 1: query i attends to keys 0..i only
  uint32_t items;    // (b, h) x query-tile groups; CTAs (groups) stride over them
  unsigned* status;
};

#ifdef FELIX_FA_TRACE
// Development-only phase trace of CTA 0 (compiled out of the library build):
// [role][block j][event] = clock64 value.
__device__ unsigned long long g_fa_trace[4][64][8];
#define FA_TRACE(role, j, ev)                                           \
  do {                                                                  \
    if (blockIdx.x == 0 && (j) < 64) g_fa_trace[role][j][ev] = clock64(); \
  } while (0)
#else
#define FA_TRACE(role, j, ev) \
  do {                        \
  } while (0)
#endif

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 arithmetic (sm_100): two lanes of fp32 in one 64-bit register,
// one instruction for both.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo_f32(uint64_t v) {
  return __uint_as_float(static_cast<uint32_t>(v));
}
__device__ __forceinline__ float hi_f32(uint64_t v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

#ifndef FELIX_FA_WAIT_PV
#define FELIX_FA_WAIT_PV 0
#endif
// 1: S_t(j+1) is issued only after PV_t(j) has completed. 0: it is issued
// right behind PV_t(j); tcgen05.mma operations of a CTA execute in issue
// order, so the later MMA's accumulator writes to S_t cannot overtake the
// earlier MMA's reads of P_t from the same columns.
constexpr int kWaitPV = FELIX_FA_WAIT_PV;
// Smem descriptor of a K-major ROWS x D tile (chunks of 64 columns, ROWS*128
// bytes each), advanced to K step k (16 elements).
template <int ROWS>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int k) {
  const uint32_t chunk = uint32_t(k) >> 2;
  return make_sdesc_sw128(tile_addr + chunk * (ROWS * 128) + (uint32_t(k) & 3u) * 32, 16, 1024);
}
// Smem descriptor of V (kBlockKV keys x its D columns, D contiguous, chunks of
// 64 columns) as the MN-major B operand of PV, advanced to K step k (16 keys).
__device__ __forceinline__ uint64_t vmajor_desc(uint32_t tile_addr, int k) {
  return make_sdesc_sw128(tile_addr + uint32_t(k) * 2048, kBlockKV * 128, 1024);
}

template <int D, int CG>
__global__ void __launch_bounds__(kThreads, 1)
    flash_attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C_ = Cfg<D, CG>;
  constexpr int KST = C_::kKStages;
  constexpr int VST = C_::kVStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_::kBarOff);
  uint64_t* q_full = bars;                   // [1]   (leader's counts both CTAs)
  uint64_t* k_full = q_full + 1;             // [KST] (leader's counts both CTAs)
  uint64_t* k_empty = k_full + KST;          // [KST]
  uint64_t* v_full = k_empty + KST;          // [VST] (leader's counts both CTAs)
  uint64_t* v_empty = v_full + VST;          // [VST]
  uint64_t* s_full = v_empty + VST;          // [2]
  uint64_t* p_full = s_full + 2;             // [2 tiles][2 halves] (leader's counts both CTAs)
  uint64_t* pv_done = s_full + 6;            // [2]
  uint64_t* drain = s_full + 8;              // [1]
  uint64_t* q_empty = s_full + 9;            // [1] Q of the current item consumed (MMA commit)
  uint64_t* o_free = s_full + 10;            // [2] O_t read out by the epilogue (leader's)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = threadIdx.x / 32;
  const uint32_t lane = threadIdx.x % 32;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  // Work items: (b, h) x group of query tiles. A CTA (group) takes items
  // first, first + stride, ...: one item when the grid has one CTA (group)
  // per item, several when the launch is persistent (one CTA per SM). Every
  // role walks the same items and counts KV blocks globally across them (jg),
  // so ring stages and barrier parities simply continue from item to item.
  const uint32_t first_item = blockIdx.x / CG, item_stride = gridDim.x / CG;
  struct Item {
    uint32_t bh, grp_q0, q0, n;
  };
  auto item_of = [&](uint32_t grp) {
    Item r;
    r.bh = grp / p.q_tiles;
    // Causal: the longest query tiles first (they bound the tail of the grid).
    const uint32_t qt = p.causal ? p.q_tiles - 1 - grp % p.q_tiles : grp % p.q_tiles;
    r.grp_q0 = qt * (2 * kBlockQ * CG);
    r.q0 = r.grp_q0 + rank * (2 * kBlockQ);
    // KV blocks this item streams: all, or (causal) up to the block that holds
    // the group's last query row. Every role of the group uses the same n.
    r.n = p.causal ? min(p.n_kv, (r.grp_q0 + 2 * kBlockQ * CG - 1) / kBlockKV + 1) : p.n_kv;
    return r;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[2 * i], 4 * CG);
      mbar_init(&p_full[2 * i + 1], 4 * CG);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(q_empty, 1);
    mbar_init(&o_free[0], 4 * CG);
    mbar_init(&o_free[1], 4 * CG);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if constexpr (CG == 2) cluster_sync();  // peer barriers initialised before any remote use
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Barrier address the loads of this CTA signal (the leader's in a pair).
  auto leader_bar = [&](uint64_t* bar) -> uint32_t {
    return CG == 2 ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar);
  };
  auto load3d = [&](void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
    if constexpr (CG == 2)
      tma_load_3d_pair(dst, map, leader_bar(bar), x, y, z);
    else
      tma_load_3d(dst, map, bar, x, y, z);
  };

  if (warp == 0 || warp == 2) {
    if constexpr (kRegSplit) setmaxnreg_dec<kRegsSide>();
    // ------------------------------------------------- loaders: warp 0 Q + K, warp 2 V
    if (elect_one()) {
      const bool is_k = warp == 0;
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      const int NS = is_k ? KST : VST;
      const uint32_t slot_bytes = is_k ? C_::kKBytes : C_::kVBytes;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* ring = smem + (is_k ? C_::kKOff : C_::kVOff);
      uint32_t filled = 0, jg = 0, ii = 0, q_issued = 0;
      bool ok = true;
      for (uint32_t it = first_item; ok && it < p.items; it += item_stride, ++ii) {
        const Item w = item_of(it);
        if (is_k) {
          // Q of the previous item must have been consumed by its S MMAs
          if (ii > 0 &&
              !(ok = mbar_wait(q_empty, (ii - 1) & 1u, abort_flag, p.status, kWdAttnLoad)))
            break;
          uint8_t* sq = smem + C_::kQOff;
          if (rank == 0) mbar_arrive_expect_tx(q_full, CG * 2 * C_::kTileBytes);
#pragma unroll
          for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int c = 0; c < C_::kChunks; ++c)
              load3d(sq + t * C_::kTileBytes + c * (kBlockQ * 128), &tmQ, q_full, 64 * c,
                     int(w.q0 + t * kBlockQ), int(w.bh));
          ++q_issued;
        }
        for (uint32_t j = 0; j < w.n; ++j, ++jg) {
          const uint32_t st = jg % NS;
          const uint32_t ph = (jg / NS) & 1u;
          if (!(ok = mbar_wait(&empty[st], ph ^ 1u, abort_flag, p.status, kWdAttnLoad))) break;
          FA_TRACE(3, j, is_k ? 3 : 2);
          uint8_t* dst = ring + st * slot_bytes;
          if (rank == 0) mbar_arrive_expect_tx(&full[st], CG * slot_bytes);
          if (is_k) {
            // K rows [key0, key0 + kKeys) of block j, all D columns
            const int key0 = int(j * kBlockKV + rank * C_::kKeys);
#pragma unroll
            for (int c = 0; c < C_::kChunks; ++c)
              load3d(dst + c * (C_::kKeys * 128), map, &full[st], 64 * c, key0, int(w.bh));
          } else {
            // all keys of block j, D columns [col0, col0 + kVCols)
            const int col0 = int(rank * C_::kVCols);
#pragma unroll
            for (int c = 0; c < C_::kVCols / 64; ++c)
              load3d(dst + c * (kBlockKV * 128), map, &full[st], col0 + 64 * c,
                     int(j * kBlockKV), int(w.bh));
          }
          ++filled;
        }
      }
      // drain: the last fill of each stage (and the last Q) must land before
      // the CTA exits; the leader's barriers count the bytes of both CTAs
      if (rank == 0) {
        int dummy = 0;
        if (is_k && q_issued > 0)
          mbar_wait(q_full, (q_issued - 1) & 1u, &dummy, p.status, kWdDrain, 100000000ull);
        const uint32_t m = filled < uint32_t(NS) ? filled : uint32_t(NS);
        for (uint32_t i = 0; i < m; ++i) {
          const uint32_t f = filled - 1 - i;
          mbar_wait(&full[f % NS], (f / NS) & 1u, &dummy, p.status, kWdDrain, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if constexpr (kRegSplit) setmaxnreg_dec<kRegsSide>();
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop (waits, descriptor arithmetic) converged;
    // one elected lane issues the MMAs and commits.
    if (rank == 0) {
      const uint32_t idesc_qk = make_idesc_f16_f32(kBlockQ * CG, kBlockKV, false, false);
      const uint32_t idesc_pv = make_idesc_f16_f32(kBlockQ * CG, D, false, true);
      const uint32_t sq = smem_u32(smem + C_::kQOff);
      auto commit_all = [&](uint64_t* bar) {
        if constexpr (CG == 2) {
          const uint32_t a = smem_u32(bar);
          umma_commit_pair(a);
          umma_commit_pair(mapa_shared(a, 1));
        } else {
          umma_commit(bar);
        }
      };
      // every lane waits and the lanes agree, so the warp stays converged
      // even when a wait gives up
      auto wait_all = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu,
                          mbar_wait(bar, parity, abort_flag, p.status, kWdAttnMma)) != 0;
      };
      bool ok = true;
      auto issue_s = [&](uint32_t j, int t) {
        const uint32_t sk = smem_u32(smem + C_::kKOff + (j % KST) * C_::kKBytes);
        const uint32_t qa = sq + t * C_::kTileBytes;
        FA_TRACE(3, j, 6 + t);
        if (elect_one()) {
          // descriptors of K step k = step 0's plus the byte offset / 16 (the
          // start-address field holds any shared-memory address + offset here)
          const uint64_t a0 = kmajor_desc<kBlockQ>(qa, 0);
          const uint64_t b0 = kmajor_desc<C_::kKeys>(sk, 0);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t ad = a0 + uint64_t(((k >> 2) * (kBlockQ * 128) + (k & 3) * 32) >> 4);
            const uint64_t bd = b0 + uint64_t(((k >> 2) * (C_::kKeys * 128) + (k & 3) * 32) >> 4);
            if constexpr (CG == 2)
              umma_f16_ss_pair(tmem + col_s(t), ad, bd, idesc_qk, k > 0 ? 1u : 0u);
            else
              umma_f16_ss(tmem + col_s(t), ad, bd, idesc_qk, k > 0 ? 1u : 0u);
          }
          commit_all(&s_full[t]);
          if (t == 1) commit_all(&k_empty[j % KST]);  // K_j consumed by both tiles
        }
        __syncwarp();
        FA_TRACE(3, j, 4 + t);
      };
      // PV_t(j) over keys [64 h, 64 h + 64): P's half h
      auto issue_pv = [&](uint32_t j, uint32_t jl, int t, int h) {
        const uint32_t sv = smem_u32(smem + C_::kVOff + (j % VST) * C_::kVBytes);
        if (elect_one()) {
          const uint64_t v0 = vmajor_desc(sv, 0);
#pragma unroll
          for (int k = h * (kBlockKV / 32); k < (h + 1) * (kBlockKV / 32); ++k) {
            const uint32_t a = tmem + col_s(t) + k * 8;
            const uint64_t vd = v0 + uint64_t(k * (2048 >> 4));
            if constexpr (CG == 2)
              umma_f16_ts_pair(tmem + col_o(t), a, vd, idesc_pv, (jl > 0 || k > 0) ? 1u : 0u);
            else
              umma_f16_ts(tmem + col_o(t), a, vd, idesc_pv, (jl > 0 || k > 0) ? 1u : 0u);
          }
          if (h == 1) {
            commit_all(&pv_done[t]);
            if (t == 1) commit_all(&v_empty[j % VST]);  // V_j consumed by both tiles
          }
        }
        __syncwarp();
      };
      // Per item: Q ready, S_A(0), S_B(0); then per block j and tile t:
      // PV_t(j) as soon as P_t(j) is ready, then S_t(j+1) right behind it
      // (the tensor pipe executes the MMAs in issue order, so S_t(j+1)'s
      // writes cannot overtake PV_t(j)'s reads of P_t). The two tiles run half
      // a period apart, so the softmax of one tile overlaps the other tile's
      // MMAs. Across items: the first PV of a tile waits until the epilogue
      // has read O_t out (o_free); Q is released once the item's S MMAs are
      // done (q_empty), so the loader can bring the next item's Q.
      uint32_t jg = 0, ii = 0;
      for (uint32_t it = first_item; ok && it < p.items; it += item_stride, ++ii) {
        const Item w = item_of(it);
        if (!(ok = wait_all(q_full, ii & 1u))) break;
        if (!(ok = wait_all(&k_full[jg % KST], (jg / KST) & 1u))) break;
        tc_fence_after();
        issue_s(jg, 0);
        issue_s(jg, 1);
        // Q is free once the item's last S MMAs complete: release it right
        // behind them, so the next item's Q loads during this item's tail
        auto release_q = [&]() {
          if (elect_one()) commit_all(q_empty);
          __syncwarp();
        };
        if (w.n == 1) release_q();
        for (uint32_t j = 0; ok && j < w.n; ++j) {
          const uint32_t g = jg + j;
          FA_TRACE(3, j, 0);
          if (!(ok = wait_all(&v_full[g % VST], (g / VST) & 1u))) break;
          FA_TRACE(3, j, 1);
          for (int t = 0; t < 2; ++t) {
            FA_TRACE(2, j, 4 * t + 0);
            if (j == 0 && ii > 0 && !(ok = wait_all(&o_free[t], (ii - 1) & 1u))) break;
            // P_t(j) arrives in two halves of 64 keys: PV over the first half
            // overlaps the softmax of the second
            if (!(ok = wait_all(&p_full[2 * t], g & 1u))) break;
            tc_fence_after();
            FA_TRACE(2, j, 4 * t + 1);
            issue_pv(g, j, t, 0);
            if (!(ok = wait_all(&p_full[2 * t + 1], g & 1u))) break;
            tc_fence_after();
            issue_pv(g, j, t, 1);
            if (j + 1 < w.n) {
              FA_TRACE(2, j, 4 * t + 2);
              if (t == 0 && !(ok = wait_all(&k_full[(g + 1) % KST], ((g + 1) / KST) & 1u)))
                break;
              if (kWaitPV && !(ok = wait_all(&pv_done[t], g & 1u))) break;
              tc_fence_after();
              FA_TRACE(2, j, 4 * t + 3);
              issue_s(g + 1, t);
              if (t == 1 && j + 2 == w.n) release_q();
            }
          }
        }
        if (!ok) break;
        jg += w.n;
      }
      if (elect_one()) {
        if constexpr (CG == 2)
          umma_commit_pair(smem_u32(drain));
        else
          umma_commit(drain);
      }
      __syncwarp();
      int dummy = 0;
      mbar_wait(drain, 0, &dummy, p.status, kWdDrain, 100000000ull);
    }
  } else if (warp == 3) {
    if constexpr (kRegSplit) setmaxnreg_dec<kRegsSide>();
  } else if (warp >= 4) {
    if constexpr (kRegSplit) setmaxnreg_inc<kRegsSoftmax>();
    // ---------------------------------------------------------------- softmax
    const int t = warp >= 8 ? 1 : 0;
    const uint32_t q = warp & 3u;
    const uint32_t row = q * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_addr = (q * 32u) << 16;
    const uint32_t tS = tmem + lane_addr + col_s(t);
    const uint32_t tO = tmem + lane_addr + col_o(t);
    const float sl2 = p.scale_log2;
    bool ok = true;
    uint32_t jg = 0;
    for (uint32_t it = first_item; ok && it < p.items; it += item_stride) {
    const Item w = item_of(it);
    const uint32_t n = w.n, q0 = w.q0, bh = w.bh;
    float m = -INFINITY;  // running max in log2 units (the one P is relative to)
    float l = 0.f;
    for (uint32_t j = 0; j < n; ++j) {
      const uint32_t g = jg + j;  // block count across items (barrier parities)
      if (lane == 0 && q == 0) FA_TRACE(t, j, 0);
      if (!(ok = mbar_wait(&s_full[t], g & 1u, abort_flag, p.status, kWdAttnSoftmax))) break;
      tc_fence_after();
      if (lane == 0 && q == 0) FA_TRACE(t, j, 1);
      // keys of this block the row may see: the ragged tail of the sequence
      // and, when causal, keys past the row's own position are masked
      uint32_t valid = p.S - j * kBlockKV;
      if (p.causal) {
        const uint32_t qrow = q0 + t * kBlockQ + row;
        const uint32_t upto = qrow + 1 > j * kBlockKV ? qrow + 1 - j * kBlockKV : 0u;
        valid = min(valid, upto);
      }
      const bool ragged = __any_sync(0xffffffffu, valid < uint32_t(kBlockKV)) != 0;
      // S is held 64 keys at a time (half h of the block), so the registers
      // left over give the exponential phase room to overlap its MUFU work
      constexpr int kHalf = kBlockKV / 2;
      float s[kHalf];                       // keys of the half being exponentiated
      float s_hi[kRegSplit ? kHalf : 1];    // register split: the second half, held
      auto load_half = [&](float* dst, int h) {  // issues the loads; tmem_ld_wait() completes them
#pragma unroll
        for (int c = 0; c < kHalf; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tS + h * kHalf + c, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) dst[c + i] = __uint_as_float(r[i]);
        }
      };
      auto mask_half = [&](float* v, int h) {
        if (ragged) {
#pragma unroll
          for (int i = 0; i < kHalf; ++i)
            if (uint32_t(h * kHalf + i) >= valid) v[i] = -INFINITY;
        }
      };
      auto max_half = [&](const float* v) -> float {  // 3-input max, 4 independent chains
        float m4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
        for (int i = 4; i < kHalf; i += 8) {
#pragma unroll
          for (int c = 0; c < 4; ++c) m4[c] = fmax3(m4[c], v[i + c], v[i + 4 + c]);
        }
        return fmax3(fmaxf(m4[0], m4[1]), m4[2], m4[3]);
      };
      // P = 2^(s * scale_log2 - m) for the keys of half h, two columns at a
      // time in packed fp32x2, exponentials on MUFU, stored as fp16 pairs over
      // the first half of S's columns
      const uint64_t scale2 = pack_f32x2(sl2, sl2);
      uint64_t l2[2] = {0ull, 0ull};  // packed partial row sums
      auto exp_half = [&](const float* v, int h) {
        const uint64_t negm2 = pack_f32x2(-m, -m);
#pragma unroll
        for (int c = 0; c < kHalf; c += 32) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = c + 2 * i;
            const uint64_t x2 = ffma2(pack_f32x2(v[e], v[e + 1]), scale2, negm2);
            const uint64_t p2 = pack_f32x2(ex2(lo_f32(x2)), ex2(hi_f32(x2)));
            l2[i & 1] = fadd2(l2[i & 1], p2);
            pk[i] = pack_half2(lo_f32(p2), hi_f32(p2));
          }
          tmem_st_32x32b_x16(tS + (h * kHalf + c) / 2, pk);
        }
      };
      auto publish = [&](int h) {
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 2)
            mbar_arrive_cluster(leader_bar(&p_full[2 * t + h]));
          else
            mbar_arrive(&p_full[2 * t + h]);
        }
      };
      // the second half's max first, then the first half, whose exponentials
      // are computed against the current running max while its own max forms
      // (the two are independent, so they interleave); they are recomputed
      // only when the max grows past the threshold (always for the first
      // block, where m is -inf and these values are discarded)
      float mx1;
      if constexpr (kRegSplit) {
        load_half(s_hi, 1);
        load_half(s, 0);
        tmem_ld_wait();
        mask_half(s_hi, 1);
        mask_half(s, 0);
        mx1 = max_half(s_hi);
      } else {
        load_half(s, 1);
        tmem_ld_wait();
        mask_half(s, 1);
        mx1 = max_half(s);
        load_half(s, 0);
        tmem_ld_wait();
        mask_half(s, 0);
      }
      if (lane == 0 && q == 0) FA_TRACE(t, j, 2);
      exp_half(s, 0);
      const float mc = fmaxf(max_half(s), mx1) * sl2;
      if (lane == 0 && q == 0) FA_TRACE(t, j, 3);
      const bool need = mc > m + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mc : m;
        const float alpha = ex2(m - m_new);  // 0 when m == -inf
        l *= alpha;
        m = m_new;
        if (j > 0) {
          // O_t holds PV(0..j-1): rescale it once PV(j-1) has completed.
          if (!(ok = mbar_wait(&pv_done[t], (g - 1) & 1u, abort_flag, p.status,
                               kWdAttnCorrection)))
            break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D; c += 16) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(tO + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st_32x32b_x16(tO + c, r);
          }
        }
        // the speculative stores must land before their replacements (stores
        // to the same TMEM columns are not ordered among themselves)
        tmem_st_wait();
        l2[0] = l2[1] = 0ull;
        exp_half(s, 0);
      }
      if constexpr (kRegSplit) {
        publish(0);
        exp_half(s_hi, 1);
      } else {
        load_half(s, 1);  // columns 64..127: untouched by P and by PV
        publish(0);
        tmem_ld_wait();
        mask_half(s, 1);
        exp_half(s, 1);
      }
      const uint64_t lsum = fadd2(l2[0], l2[1]);
      l += lo_f32(lsum) + hi_f32(lsum);
      if (lane == 0 && q == 0) FA_TRACE(t, j, 4);
      publish(1);
      if (lane == 0 && q == 0) FA_TRACE(t, j, 5);
      if (lane == 0 && q == 0) FA_TRACE(t, j, 6);
#ifdef FELIX_FA_TRACE
      if (lane == 0 && blockIdx.x == 0 && j < 64) atomicMax(&g_fa_trace[t][j][7], clock64());
#endif
    }
    // ---------------------------------------------------------------- epilogue
    if (!ok) break;
    if (!(ok = mbar_wait(&pv_done[t], (jg + n - 1) & 1u, abort_flag, p.status,
                         kWdAttnSoftmax)))
      break;
    {
      tc_fence_after();
      const uint32_t qrow = q0 + t * kBlockQ + row;
      const float inv_l = 1.f / l;
      __half* dst = p.O + (size_t(bh) * p.S + qrow) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tO + c, r);
        tmem_ld_wait();
        if (qrow < p.S) {
          uint4 o4[4];
          uint32_t* o = reinterpret_cast<uint32_t*>(o4);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[i] = pack_half2(__uint_as_float(r[2 * i]) * inv_l,
                              __uint_as_float(r[2 * i + 1]) * inv_l);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = o4[i];
        }
      }
      if (p.lse && qrow < p.S)
        p.lse[size_t(bh) * p.S + qrow] = (m + __log2f(l)) * 0.69314718055994531f;
    }
    // O_t has been read out: the next item's first PV_t may overwrite it
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if constexpr (CG == 2)
        mbar_arrive_cluster(leader_bar(&o_free[t]));
      else
        mbar_arrive(&o_free[t]);
    }
    jg += n;
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // no remote signal may target an exited CTA
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem, 512);
    else
      tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace felix_sm100

// ============================================================ host launcher
namespace felix_impl {

using namespace felix_sm100::attn;

namespace {

// CTA-pair attention is a build option, off by default: on B200 it is exact
// (bit-identical O) but slower (4x32x8192x128: 896 vs 1148 TFLOP/s; the
// pair's cross-CTA barriers cost more than the halved K/V operand traffic saves).
#ifndef FELIX_FA_PAIRS
#define FELIX_FA_PAIRS 0
#endif
constexpr bool felix_fa_pairs_enabled() { return FELIX_FA_PAIRS != 0; }

int encode_qkv(CUtensorMap* map, const void* base, uint32_t BH, uint32_t S, uint32_t D,
               uint32_t box_rows) {
  // 3-D view [BH][S][D] so that a tile never crosses into the next head:
  // rows past S are zero-filled by the TMA unit.
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  return encode_tmap_3d_f16(map, base, D, S, BH, uint64_t(D) * 2, uint64_t(S) * D * 2, 64,
                            box_rows, 1);
}

template <int D, int CG>
int configure_once(int device) {
  static PerDeviceOnce once;
  return once.run(device, [] {
    cudaError_t e = cudaFuncSetAttribute(flash_attn_fwd_kernel<D, CG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg<D, CG>::kSmemBytes);
    if (e != cudaSuccess) return int(e);
    if (kRegSplit) {
      // the register split's arithmetic assumes the launch register count
      cudaFuncAttributes fa{};
      e = cudaFuncGetAttributes(&fa, flash_attn_fwd_kernel<D, CG>);
      if (e != cudaSuccess) return int(e);
      if (fa.numRegs != kRegsLaunch) {
        char msg[160];
        std::snprintf(msg, sizeof msg,
                      "flash_attn: the kernel was compiled with %d registers per thread, but its "
                      "setmaxnreg split assumes %d (rebuild with FELIX_FA_REGSPLIT=0)",
                      fa.numRegs, kRegsLaunch);
        api_error(msg, cudaErrorInvalidConfiguration);
        return -2;
      }
    }
    return 0;
  });
}

FelixCode configure_error(int rc) {
  if (rc == -2) return FelixCode{FELIX_API_ERROR, cudaErrorInvalidConfiguration};  // message set
  return api_error("flash_attn: kernel set-up (cudaFuncSetAttribute) failed",
                   rc > 0 ? cudaError_t(rc) : cudaErrorInvalidDevice);
}

template <int D, int CG>
cudaError_t launch(uint64_t groups, const CUtensorMap& tq, const CUtensorMap& tk,
                   const CUtensorMap& tv, const Params& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(unsigned(groups * CG), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg<D, CG>::kSmemBytes;
  cfg.stream = stream;
  if (CG == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, flash_attn_fwd_kernel<D, CG>, tq, tk, tv, p);
}

}  // namespace

FelixCode flash_attn_launch(const __half* Q, const __half* K, const __half* V, __half* O,
                            float* lse, uint32_t heads, uint32_t batch, uint32_t seqlen,
                            uint32_t head_dim, float scale, bool causal, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128)
    return api_error("flash_attn: head_dim must be 64 or 128");
  if (heads == 0 || batch == 0 || seqlen == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  if (!Q || !K || !V || !O) return api_error("flash_attn: null pointer");
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
       reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(O)) & 15u)
    return api_error("flash_attn: Q, K, V, O must be 16-byte aligned");
  const uint64_t bh = uint64_t(heads) * batch;
  if (bh > (1u << 31) || seqlen > (1u << 30)) return api_error("flash_attn: problem too large");
  DeviceInfo* dev = current_device_info();
  if (!dev) return launch_error(cudaGetLastError(), "flash_attn: no CUDA device");

  // CTA pairs (D = 128) once a head has at least 512 query rows.
  const int cg = (head_dim == 128 && seqlen >= 512 && felix_fa_pairs_enabled()) ? 2 : 1;
  CUtensorMap tq, tk, tv;
  if (encode_qkv(&tq, Q, uint32_t(bh), seqlen, head_dim, kBlockQ) ||
      encode_qkv(&tk, K, uint32_t(bh), seqlen, head_dim, kBlockKV / cg) ||
      encode_qkv(&tv, V, uint32_t(bh), seqlen, head_dim, kBlockKV))
    return api_error("flash_attn: cuTensorMapEncodeTiled failed");

  Params p{};
  p.O = O;
  p.lse = lse;
  p.S = seqlen;
  p.n_kv = (seqlen + kBlockKV - 1) / kBlockKV;
  p.causal = causal ? 1u : 0u;
  p.q_tiles = (seqlen + 2 * kBlockQ * cg - 1) / (2 * kBlockQ * cg);
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf(float(head_dim));
  p.scale_log2 = sc * 1.4426950408889634f;
  p.status = dev->status_word;
  const uint64_t groups = bh * p.q_tiles;
  if (groups * cg > 0x7fffffffull) return api_error("flash_attn: grid too large");
  p.items = uint32_t(groups);
  // Persistent (one CTA per SM walking the items) when there are more items
  // than SMs and every item is the same length; causal items differ, so they
  // keep one CTA per item, longest first.
  const uint64_t grid_groups =
      (cg == 1 && !causal && groups > uint64_t(dev->num_sms)) ? uint64_t(dev->num_sms) : groups;

  int rc;
  cudaError_t e;
  if (head_dim == 128 && cg == 2) {
    if ((rc = configure_once<128, 2>(dev->ordinal))) return configure_error(rc);
    e = launch<128, 2>(grid_groups, tq, tk, tv, p, stream);
  } else if (head_dim == 128) {
    if ((rc = configure_once<128, 1>(dev->ordinal))) return configure_error(rc);
    e = launch<128, 1>(grid_groups, tq, tk, tv, p, stream);
  } else {
    if ((rc = configure_once<64, 1>(dev->ordinal))) return configure_error(rc);
    e = launch<64, 1>(grid_groups, tq, tk, tv, p, stream);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return launch_error(e, "flash_attn: launch failed");
  return FelixCode{FELIX_SUCCESS, cudaSuccess};
}

}  // namespace felix_impl

#ifdef FELIX_FA_TRACE
extern "C" void fa_trace_fetch(void* dst) {
  cudaMemcpyFromSymbol(dst, felix_sm100::attn::g_fa_trace, sizeof(felix_sm100::attn::g_fa_trace));
}
#endif
