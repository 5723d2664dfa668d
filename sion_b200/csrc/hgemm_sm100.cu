// HGEMM for sm_100a: C = alpha * A * op(B) + beta * C, fp16 in, fp32 accumulate
// (TMEM), fp16 out. Replaces the Ampere mma.sync kernel behind
// felix::ampere_hgemm_launch (reference: src/felix/gemm/hgemm/
// cute_hgemm_128x128_{nn,nt}_kernel_launch.cu, kernels/cute_ampere_hgemm_16816.cuh),
// which accumulates in fp16; this one accumulates in fp32.
//
// Layouts (all row-major, as in the reference):
//   A [M x K]; "nt": B stored [N x K] (K-major); "nn": B stored [K x N] (N-major);
//   C [M x N].
//
// Design:
//   * persistent grid, one CTA per SM, 6 warps:
//       warp 0  TMA producer (one elected lane), multi-stage smem ring
//       warp 1  TMEM allocator + single-thread tcgen05.mma issuer
//       warps 2-5 epilogue: tcgen05.ld -> alpha/beta -> fp16 -> global
//   * CTA tile 128 x BN (BN = 256, 128 or 64; CTA pairs 256 x 256 or, for many
//     waves of "nt" tiles, 256 x 512 from two N = 256 MMAs per k step into a
//     single TMEM accumulator), K step 64 (one 128-byte swizzle row),
//     UMMA 128 x BN x 16; two TMEM accumulators so the epilogue of tile i
//     overlaps the main loop of tile i+1.
//   * schedule: whole tiles over the persistent CTAs ("data-parallel" waves),
//     in a grouped raster; with four or more waves the tiles are handed out at
//     run time from a global counter (TileQueue), so the CTAs running together
//     always share operand panels in L2; the tiles of an incomplete last wave are spread evenly over all
//     CTAs by k-iterations (stream-K). A stream-K tile with several contributors
//     is finished by whichever contributor arrives last (atomic ticket): every
//     contributor writes its fp32 partial to the workspace, the last one sums all
//     partials in contributor order (deterministic) and writes C. No CTA ever
//     waits on another CTA.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "felix_internal.h"
#include "sm100_ptx.cuh"

namespace felix_sm100 {
namespace hgemm {

constexpr int BM = 128;
// K step of one pipeline stage: 64 (128-byte operand rows, SWIZZLE_128B).
// 32 (SWIZZLE_64B, twice as many half-size stages) is kept as a build option;
// measured on B200 it is slower (4096^3: 1005 vs 1335 TFLOP/s) because the
// per-stage barrier and issue work doubles.
#ifndef FELIX_HGEMM_BK
#define FELIX_HGEMM_BK 64
#endif
constexpr int BK = FELIX_HGEMM_BK;
static_assert(BK == 32 || BK == 64, "k step");
constexpr int kSwizzleK = BK * 2;  // bytes per K-major operand row = swizzle span
constexpr int kThreads = 192;

// CG = 2: CTA pairs (cta_group::2): a 2-CTA cluster computes a 256 x BN tile;
// each CTA holds 128 rows of A and BN / 2 rows (N) of B, the leader issues the
// MMAs (M = 256) and each CTA's TMEM gets its own 128 rows of the tile.
// A pair's stages hold two 64-deep k-blocks, loaded by one 32 KB TMA request
// per operand (3-D tensor-map view): requests of 16 KB stream at only ~57
// B/clk per SM from L2 against ~90 for 32 KB ones, and the pair needs ~63.
template <int BN, int CG = 1, int SUB = (CG == 2 ? 2 : 1)>
struct Cfg {
  static_assert(CG == 1 || SUB == 2 || BN == 512, "CTA pairs load two k-blocks per stage");
  static constexpr int kBRows = BN / CG;  // B rows (N) loaded by one CTA
  // BN = 512 (CTA pairs only): two N = 256 MMAs per k step, each CTA holding
  // 128 B rows of each half; one accumulator (all 512 TMEM columns)
  static constexpr int kNH = BN > 256 ? 2 : 1;        // MMA N halves
  static constexpr int kBoxRows = kBRows / kNH;        // B rows per load box
  static constexpr int kNBuf = 2 * BN <= 512 ? 2 : 1;  // TMEM accumulators
  static constexpr int kSub = SUB;        // 64-deep k-blocks per stage
  static constexpr int kStages = (192 * 1024) / ((BM + kBRows) * BK * 2 * kSub);
  static constexpr int kABytes = BM * BK * 2 * kSub;
  static constexpr int kBBytes = kBRows * BK * 2 * kSub;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = kNBuf * BN;
  // epilogue staging for TMA stores: 4 warps x 2 buffers x (32 rows x 128 B)
  static constexpr int kStagingBytes = 4 * 2 * 4096;
  // ring + staging + 1 KB alignment slack + barrier block
  static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 + 512;
};

struct Params {
  uint32_t M, N, K;
  float alpha, beta;
  __half* C;
  uint32_t b_mn_major;  // 1 = "nn" (B is K x N), 0 = "nt" (B is N x K)
  uint32_t tiles_m, tiles_n, kblocks;
  uint32_t dp_tiles, sk_tiles;
  uint64_t sk_iters;
  uint32_t sk_units;      // units (CTAs or pairs) sharing the stream-K iterations (<= grid)
  uint32_t group_m;
  uint32_t tma_store;     // 1: epilogue writes C through smem + TMA (beta == 0)
  uint32_t ksplit2;       // 1: 2-CTA clusters split each tile's K in halves (see below)
  uint32_t pair;          // 1: CTA pairs (cta_group::2); units and slots are per pair
  uint32_t dyn;           // 1: whole tiles are handed out at run time (see TileQueue)
  unsigned* ws_dyn;       // [0] next whole tile, [1] finished leader CTAs; zero between launches
  float* ws_partials;     // [gridDim.x][2] slots of BM*BN fp32, see partial_index()
  unsigned* ws_counters;  // [sk_tiles], zero between launches
  unsigned* status;       // watchdog word
};

struct Unit {
  uint32_t tile;   // linear tile id (0..tiles-1)
  uint32_t kb0, kb1;
  uint32_t sk;     // stream-K tile index (valid when partial)
  uint32_t seg;    // 0/1: which of this CTA's two partial slots
  bool partial;
};

// Identical walk for the producer, MMA and epilogue roles of one CTA.
// Stream-K units come first (tiles [0, sk_tiles) spread over all CTAs by
// k-iterations), then whole tiles sk_tiles + cta + i * P. Doing the split tiles
// first lets their fix-up in the epilogue warps overlap the main loop of the
// following whole tiles instead of forming a tail.
struct Sched {
  uint32_t cta, P, Psk, sk_tiles, tiles, KB;
  uint64_t I, it, end, start;
  uint32_t dp_next;
  bool dyn;

  uint32_t ksplit_rank;  // cluster split-K: 0 or 1 (which half of K); 2 = unit taken
  __device__ __forceinline__ void init(const Params& p) {
    ksplit_rank = p.ksplit2 ? (blockIdx.x & 1u) : 3u;
    cta = p.pair ? blockIdx.x >> 1 : blockIdx.x;
    P = p.pair ? gridDim.x >> 1 : gridDim.x;
    sk_tiles = p.sk_tiles;
    tiles = p.sk_tiles + p.dp_tiles;
    KB = p.kblocks;
    I = p.sk_iters;
    // stream-K iterations go to the first Psk units only
    Psk = p.sk_units ? p.sk_units : P;
    start = cta < Psk ? I * cta / Psk : I;
    end = cta < Psk ? I * (cta + 1) / Psk : I;
    it = start;
    dp_next = sk_tiles + cta;
    dyn = p.dyn != 0;
  }
  // whole tile t (dynamic schedule)
  __device__ __forceinline__ void whole(Unit& u, uint32_t t) const {
    u.tile = t;
    u.kb0 = 0;
    u.kb1 = KB;
    u.partial = false;
    u.sk = 0;
    u.seg = 0;
  }
  __device__ __forceinline__ bool next(Unit& u) {
    if (ksplit_rank < 2) {
      // cluster split-K: tile blockIdx.x / 2, K half blockIdx.x % 2
      const uint32_t half = KB / 2;
      u.tile = cta >> 1;
      u.kb0 = ksplit_rank ? half : 0;
      u.kb1 = ksplit_rank ? KB : half;
      u.partial = false;
      u.sk = 0;
      u.seg = ksplit_rank;
      ksplit_rank = 2;
      return true;
    }
    if (ksplit_rank == 2) return false;
    if (it < end) {
      const uint32_t s = static_cast<uint32_t>(it / KB);
      const uint32_t kb0 = static_cast<uint32_t>(it - uint64_t(s) * KB);
      const uint64_t left = end - it;
      const uint32_t kb1 = left < uint64_t(KB - kb0) ? kb0 + static_cast<uint32_t>(left) : KB;
      u.tile = s;
      u.kb0 = kb0;
      u.kb1 = kb1;
      u.sk = s;
      u.seg = (it == start) ? 0u : 1u;
      u.partial = !(kb0 == 0 && kb1 == KB);
      it += kb1 - kb0;
      return true;
    }
    if (!dyn && dp_next < tiles) {
      u.tile = dp_next;
      u.kb0 = 0;
      u.kb1 = KB;
      u.partial = false;
      u.sk = 0;
      u.seg = 0;
      dp_next += P;
      return true;
    }
    return false;
  }
  // CTA whose k-range contains stream-K iteration `x`.
  __device__ __forceinline__ uint32_t cta_of(uint64_t x) const {
    return static_cast<uint32_t>(((x + 1) * Psk - 1) / I);
  }
};

// Dynamic whole-tile schedule (Params::dyn). With a static stride the
// persistent CTAs drift apart over many waves (16384^3: 55 waves), so the CTAs
// running at the same time stop sharing A and B panels in L2: measured 18.9 GB
// of DRAM reads for 1.07 GB of operands. Instead the leader CTA's producer
// takes each next whole tile from a global counter (one atomicAdd per tile,
// fetched one tile ahead) and hands it to every role of its CTA, and of the
// peer CTA of a pair, through a kTq-slot queue in shared memory: tq[slot],
// tq_full[slot] (completed by the producer's arrival; the peer's copy by a
// remote arrival after a remote store) and the leader's tq_empty[slot] (one
// arrival per consuming warp role, remote ones from the peer). Tiles then run
// in the order the CTAs become free: neighbours in the grouped raster run
// together. Each tile is still computed by one CTA (pair) in a fixed k order,
// so results do not depend on the assignment. A tile id >= tiles ends the walk.
constexpr uint32_t kTq = 4;
struct TileQueue {
  uint32_t* tq;
  uint64_t* full;
  uint64_t* empty;
  uint32_t n;  // queue entries used so far
};

__device__ __forceinline__ bool tq_push(TileQueue& q, uint32_t t, bool pair,
                                        volatile int* abort_flag, unsigned* status) {
  const uint32_t slot = q.n % kTq, par = (q.n / kTq) & 1u;
  if (!mbar_wait_cluster(&q.empty[slot], par ^ 1u, abort_flag, status, kWdTileQueue))
    return false;
  q.tq[slot] = t;
  if (pair) {
    st_shared_cluster_u32(mapa_shared(smem_u32(&q.tq[slot]), 1), t);
    mbar_arrive_cluster(mapa_shared(smem_u32(&q.full[slot]), 1));
  }
  mbar_arrive(&q.full[slot]);
  ++q.n;
  return true;
}

// Waits for the next queue entry and reads it (every calling thread); the
// caller then releases the slot once per warp with tq_release.
__device__ __forceinline__ bool tq_pop(TileQueue& q, uint32_t& t, uint32_t& slot,
                                       volatile int* abort_flag, unsigned* status) {
  slot = q.n % kTq;
  const uint32_t par = (q.n / kTq) & 1u;
  if (!mbar_wait_cluster(&q.full[slot], par, abort_flag, status, kWdTileQueue)) return false;
  t = reinterpret_cast<volatile uint32_t*>(q.tq)[slot];
  ++q.n;
  return true;
}

__device__ __forceinline__ void tq_release(TileQueue& q, uint32_t slot, uint32_t rank) {
  if (rank == 0)
    mbar_arrive(&q.empty[slot]);
  else
    mbar_arrive_cluster(mapa_shared(smem_u32(&q.empty[slot]), 0));
}

__device__ __forceinline__ void tile_coords(const Params& p, uint32_t t, uint32_t& tm,
                                            uint32_t& tn) {
  // Grouped raster: runs of group_m M-tiles sweep across N, so CTAs running at
  // the same time share A row-panels and B column-panels in L2.
  const uint32_t per_group = p.group_m * p.tiles_n;
  const uint32_t g = t / per_group;
  const uint32_t first_m = g * p.group_m;
  const uint32_t gm = min(p.group_m, p.tiles_m - first_m);
  const uint32_t r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

// Float4 index of (chunk c of 32 columns, float4 j within the chunk, row r) in
// a partial-tile slot: a warp's 32 rows touch 512 contiguous bytes.
__device__ __forceinline__ uint32_t partial_index(uint32_t c, uint32_t j, uint32_t r) {
  return (c * 8u + j) * BM + r;
}

// Convert 32 fp32 accumulators (columns c..c+31 of row `row`) and store to C.
__device__ __forceinline__ void store_row_chunk(const Params& p, uint32_t row, uint32_t col,
                                                const float (&v)[32]) {
  if (row >= p.M) return;
  __half* dst = p.C + size_t(row) * p.N + col;
  const bool full = (col + 32 <= p.N) && ((p.N & 7u) == 0);
  if (full) {
    uint4 out[4];
    uint32_t* o = reinterpret_cast<uint32_t*>(out);
    if (p.beta != 0.f) {
      uint4 old[4];
      const uint4* src = reinterpret_cast<const uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i) old[i] = src[i];
      const __half2* oh = reinterpret_cast<const __half2*>(old);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 c = __half22float2(oh[i]);
        o[i] = pack_half2(fmaf(p.alpha, v[2 * i], p.beta * c.x),
                          fmaf(p.alpha, v[2 * i + 1], p.beta * c.y));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = pack_half2(p.alpha * v[2 * i], p.alpha * v[2 * i + 1]);
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d4[i] = out[i];
  } else {
    for (int i = 0; i < 32; ++i) {
      if (col + i < p.N) {
        float r = p.alpha * v[i];
        if (p.beta != 0.f) r = fmaf(p.beta, __half2float(dst[i]), r);
        dst[i] = __float2half_rn(r);
      }
    }
  }
}

#ifdef FELIX_HGEMM_TRACE
// Development-only per-CTA timeline (compiled out of the library build):
// [cta][event] = globaltimer ns.
__device__ unsigned long long g_hg_trace[1024][12];
__device__ unsigned g_hg_tiles[1024][8];
#define HG_TR(ev)                                                   \
  do {                                                              \
    if (blockIdx.x < 1024) g_hg_trace[blockIdx.x][ev] = globaltimer_ns(); \
  } while (0)
#else
#define HG_TR(ev) \
  do {            \
  } while (0)
#endif

template <int BN, int CG = 1, int SUB = (CG == 2 ? 2 : 1)>
__global__ void __launch_bounds__(kThreads, 1)
    hgemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, const Params p) {
  using C_ = Cfg<BN, CG, SUB>;
  static_assert(CG == 1 || BN == 256 || BN == 512, "CTA pairs use 256- or 512-wide tiles");
  static_assert(BN <= 256 || CG == 2, "512-wide tiles only on CTA pairs");
  static_assert(SUB == 1 || (BK == 64 && C_::kBoxRows == 128), "3-D loads: 128-row boxes, BK = 64");
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  constexpr int S = C_::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* staging = smem + S * C_::kStageBytes;  // 1 KB aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C_::kStagingBytes);
  uint64_t* full = bars;               // [S]
  uint64_t* empty = bars + S;          // [S]
  uint64_t* tfull = bars + 2 * S;      // [2]
  uint64_t* tempty = bars + 2 * S + 2; // [2]
  uint64_t* drain = bars + 2 * S + 4;  // [1]
  uint64_t* recv = bars + 2 * S + 5;   // [1] cluster split-K: the peer's half has arrived
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 7);
  const uint32_t NS = uint32_t(S);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* bcast = tmem_slot + 2;
  TileQueue tq{reinterpret_cast<uint32_t*>(bars + 2 * S + 17), bars + 2 * S + 9,
               bars + 2 * S + 13, 0};
  static_assert((2 * S + 19) * 8 <= 512, "barrier block");

  const uint32_t warp = threadIdx.x / 32;
  const uint32_t lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4 * CG);  // a pair's leader counts both CTAs' epilogue warps
    }
    mbar_init(drain, 1);
    mbar_init(recv, 128);  // one arrival per epilogue thread of the peer CTA
    for (uint32_t i = 0; i < kTq; ++i) {
      mbar_init(&tq.full[i], 1);
      // consumers: the leader's MMA warp and 4 epilogue warps; in a pair also
      // the peer's producer and 4 epilogue warps
      mbar_init(&tq.empty[i], CG == 2 ? 10 : 5);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.tma_store) tma_prefetch_desc(&tmC);
  }
  if (CG == 2 || p.ksplit2)
    cluster_sync();  // the peer uses this CTA's barriers: they must be initialised
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, C_::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C_::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) HG_TR(0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      Sched sc;
      sc.init(p);
      Unit u;
      uint32_t stage = 0, phase = 0;
      uint32_t filled = 0;
      bool ok = true;
      // loads of a pair's CTAs complete on the leader's barrier
      auto load2d = [&](void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
        if constexpr (CG == 2)
          tma_load_2d_pair(dst, map, mapa_shared(smem_u32(bar), 0), x, y);
        else
          tma_load_2d(dst, map, bar, x, y);
      };
      // two-k-block stages: 3-D views (64-element inner, rows, 64-wide k-blocks
      // or n-chunks); a pair's loads complete on the leader's barrier
      auto load3d = [&](void* dst, const CUtensorMap* map, uint64_t* bar, int y, int z) {
        if constexpr (CG == 2)
          tma_load_3d_pair(dst, map, mapa_shared(smem_u32(bar), 0), 0, y, z);
        else
          tma_load_3d(dst, map, bar, 0, y, z);
      };
      // dynamic schedule: the leader fetches tile ids one tile ahead and
      // pushes them; the peer of a pair pops them
      uint32_t ahead = 0;
      bool have_ahead = false;
      auto next_unit = [&](Unit& uu) -> bool {
        if (sc.next(uu)) return true;
        if (!sc.dyn) return false;
        uint32_t t;
        if (rank == 0) {
          if (!have_ahead) ahead = sc.sk_tiles + atomicAdd(p.ws_dyn, 1u);
          t = ahead;
          if (!tq_push(tq, t, CG == 2, abort_flag, p.status)) return ok = false;
          have_ahead = t < sc.tiles;
          if (have_ahead) ahead = sc.sk_tiles + atomicAdd(p.ws_dyn, 1u);
        } else {
          uint32_t slot;
          if (!tq_pop(tq, t, slot, abort_flag, p.status)) return ok = false;
          tq_release(tq, slot, rank);
        }
        if (t >= sc.tiles) return false;
        sc.whole(uu, t);
        return true;
      };
      while (ok && next_unit(u)) {
        uint32_t tm, tn;
        tile_coords(p, u.tile, tm, tn);
        const int m0 = int(tm * BM * CG + rank * BM), n0 = int(tn * BN + rank * C_::kBRows);
        for (uint32_t kb = u.kb0; kb < u.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, kWdProducerEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = ring + stage * C_::kStageBytes;
          uint8_t* sb = sa + C_::kABytes;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], CG * C_::kStageBytes);
          if constexpr (SUB == 2) {
            // A rows [m0, m0 + 128), k-blocks 2 kb, 2 kb + 1; B likewise, or
            // ("nn") k rows [128 kb, 128 kb + 128) of n-chunks n0 / 64, + 1
            load3d(sa, &tmA, &full[stage], m0, int(2 * kb));
            if constexpr (C_::kNH == 2) {
              // "nt" only: B rows of N half h, this CTA's 128 of them
#pragma unroll
              for (int h = 0; h < 2; ++h)
                load3d(sb + h * (C_::kBBytes / 2), &tmB, &full[stage],
                       int(tn * BN + h * (BN / 2) + rank * C_::kBoxRows), int(2 * kb));
            } else if (p.b_mn_major) {
              load3d(sb, &tmB, &full[stage], int(kb * BK * 2), n0 / 64);
            } else {
              load3d(sb, &tmB, &full[stage], n0, int(2 * kb));
            }
          } else if constexpr (C_::kNH == 2) {
            // 256 x 512 pair tiles, one 64-deep k-block per stage ("nt")
            load2d(sa, &tmA, &full[stage], int(kb * BK), m0);
#pragma unroll
            for (int h = 0; h < 2; ++h)
              load2d(sb + h * (C_::kBBytes / 2), &tmB, &full[stage], int(kb * BK),
                     int(tn * BN + h * (BN / 2) + rank * C_::kBoxRows));
          } else {
            load2d(sa, &tmA, &full[stage], int(kb * BK), m0);
            if (p.b_mn_major) {
#pragma unroll
              for (int j = 0; j < C_::kBRows / 64; ++j)
                load2d(sb + j * (64 * BK * 2), &tmB, &full[stage], n0 + 64 * j, int(kb * BK));
            } else {
              load2d(sb, &tmB, &full[stage], int(kb * BK), n0);
            }
          }
          ++filled;
          if (++stage == NS) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      HG_TR(9);
      // Drain: wait (bounded) for the last fill of every stage so that no TMA
      // write is in flight when the CTA exits (a pair's leader counts both
      // CTAs' bytes; the final cluster barrier holds the peer until then).
      const uint32_t n = rank == 0 ? (filled < NS ? filled : NS) : 0u;
      for (uint32_t i = 0; i < n; ++i) {
        // stage of the i-th most recent fill, and the phase parity it filled
        const uint32_t f = filled - 1 - i;
        const uint32_t st = f % NS;
        const uint32_t par = (f / NS) & 1u;
        int dummy = 0;
        mbar_wait(&full[st], par, &dummy, p.status, kWdDrain, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // a pair's leader issues for both CTAs. The whole warp runs the loop
    // converged (every lane waits, the lanes agree on the outcome); one
    // elected lane issues the MMAs and commits.
    if (rank == 0) {
      auto wait_all = [&](uint64_t* bar, uint32_t parity, unsigned site) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status, site)) != 0;
      };
      const uint32_t idesc =
          make_idesc_f16_f32(BM * CG, BN / C_::kNH, false, p.b_mn_major != 0);
      // completion signals go to the barrier in every CTA of the group
      auto commit_all = [&](uint64_t* bar) {
        if constexpr (CG == 2) {
          const uint32_t a = smem_u32(bar);
          umma_commit_pair(a);
          umma_commit_pair(mapa_shared(a, 1));
        } else {
          umma_commit(bar);
        }
      };
      Sched sc;
      sc.init(p);
      Unit u;
      uint32_t stage = 0, phase = 0, i = 0;
      bool ok = true;
      // dynamic schedule: every lane pops (the warp stays converged), lane 0
      // releases the slot
      auto next_unit = [&](Unit& uu) -> bool {
        if (sc.next(uu)) return true;
        if (!sc.dyn) return false;
        uint32_t t, slot;
        const bool got = tq_pop(tq, t, slot, abort_flag, p.status);
        if (__all_sync(0xffffffffu, got) == 0) return ok = false;
        __syncwarp();
        if (lane == 0) tq_release(tq, slot, 0);
        if (t >= sc.tiles) return false;
        sc.whole(uu, t);
        return true;
      };
      while (ok && next_unit(u)) {
        const uint32_t buf = C_::kNBuf == 2 ? (i & 1u) : 0u;
        const uint32_t use_par = C_::kNBuf == 2 ? ((i >> 1) & 1u) : (i & 1u);
        if (!wait_all(&tempty[buf], use_par ^ 1u, kWdMmaTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        for (uint32_t kb = u.kb0; kb < u.kb1; ++kb) {
          if (!wait_all(&full[stage], phase, kWdMmaFull)) {
            ok = false;
            break;
          }
          if (lane == 0 && i == 0 && kb == u.kb0) HG_TR(1);
          tc_fence_after();
          if (elect_one()) {
            const uint32_t a0 = smem_u32(ring + stage * C_::kStageBytes);
            const uint32_t b0 = a0 + C_::kABytes;
            // descriptors of step k = step 0's + byte offset / 16 (the
            // start-address field never carries for shared memory)
            uint64_t ad0, bd0;
            if constexpr (BK == 64) {
              ad0 = make_sdesc_sw128(a0, 16, 1024);
              bd0 = p.b_mn_major ? make_sdesc_sw128(b0, BK * C_::kSub * 128, 1024)
                                 : make_sdesc_sw128(b0, 16, 1024);
            } else {
              ad0 = make_sdesc_sw64(a0, 16, 512);
              bd0 = p.b_mn_major ? make_sdesc_sw128(b0, 64 * BK * 2, 1024)
                                 : make_sdesc_sw64(b0, 16, 512);
            }
#pragma unroll
            for (int k = 0; k < BK * C_::kSub / 16; ++k) {
              uint32_t aoff, boff;
              if constexpr (BK == 64) {
                // K-major: 64-deep k-blocks of rows x 128 B, 32 B per 16 k;
                // MN-major: 64-wide chunks of (BK * kSub) k-rows x 128 B
                constexpr int kq = BK / 16;
                aoff = (k / kq) * (BM * BK * 2) + (k % kq) * 32;
                boff = p.b_mn_major ? k * 2048 : (k / kq) * (C_::kBoxRows * BK * 2) + (k % kq) * 32;
              } else {
                aoff = k * 32;
                boff = p.b_mn_major ? k * 2048 : k * 32;
              }
              const uint64_t ad = ad0 + (aoff >> 4), bd = bd0 + (boff >> 4);
#pragma unroll
              for (int h = 0; h < C_::kNH; ++h) {
                // N half h: its B box follows the previous one in the stage
                const uint64_t bdh = bd + uint64_t(h * (C_::kBBytes / C_::kNH) >> 4);
                const uint32_t dh = d + uint32_t(h * (BN / C_::kNH));
                if constexpr (CG == 2)
                  umma_f16_ss_pair(dh, ad, bdh, idesc, (kb > u.kb0 || k > 0) ? 1u : 0u);
                else
                  umma_f16_ss(dh, ad, bdh, idesc, (kb > u.kb0 || k > 0) ? 1u : 0u);
              }
            }
            commit_all(&empty[stage]);
          }
          __syncwarp();
          if (++stage == NS) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) commit_all(&tfull[buf]);
        if (lane == 0) HG_TR(2);
#ifdef FELIX_HGEMM_TRACE_UNITS
        if (lane == 0 && i < 5) HG_TR(3 + i);
        if (lane == 0 && i == 0) g_hg_trace[blockIdx.x < 1024 ? blockIdx.x : 0][11] = u.partial ? 1000u + u.kb1 - u.kb0 : u.kb1 - u.kb0;
        if (lane == 0 && i < 8 && blockIdx.x < 1024) g_hg_tiles[blockIdx.x][i] = (u.partial ? 0x80000000u : 0u) | u.tile;
#endif
        __syncwarp();
        ++i;
      }
      // Wait (bounded) until every issued MMA has completed before teardown.
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
  } else {
    // ------------------------------------------------------------ epilogue
    const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
    const uint32_t row_in_tile = q * 32 + lane;
    const uint32_t epi_tid = threadIdx.x - 64;  // 0..127
    Sched sc;
    sc.init(p);
    Unit u;
    uint32_t i = 0;
    auto next_unit = [&](Unit& uu) -> bool {
      if (sc.next(uu)) return true;
      if (!sc.dyn) return false;
      uint32_t t, slot;
      if (!tq_pop(tq, t, slot, abort_flag, p.status)) return false;
      __syncwarp();
      if (lane == 0) tq_release(tq, slot, rank);
      if (t >= sc.tiles) return false;
      sc.whole(uu, t);
      return true;
    };
    while (next_unit(u)) {
      const uint32_t buf = C_::kNBuf == 2 ? (i & 1u) : 0u;
      const uint32_t use_par = C_::kNBuf == 2 ? ((i >> 1) & 1u) : (i & 1u);
      if (!mbar_wait(&tfull[buf], use_par, abort_flag, p.status, kWdEpilogueTmemFull))
        break;
      tc_fence_after();
      uint32_t tm, tn;
      tile_coords(p, u.tile, tm, tn);
      const uint32_t row0 = tm * BM * CG + rank * BM;  // this CTA's first row of the tile
      const uint32_t row = row0 + row_in_tile;
      const uint32_t col0 = tn * BN;
      const uint32_t taddr = tmem_base + ((q * 32u) << 16) + buf * BN;

      if (p.ksplit2) {
        // Cluster split-K: the two CTAs hold the tile's two K halves. Rank r
        // writes output columns [64 r, 64 r + 64): as soon as its own MMAs
        // have completed it sends the peer's 64 columns of its fp32
        // accumulator over DSMEM into the peer's epilogue staging area (warp
        // q's 32 rows fill warp q's 8 KB there, 512 contiguous bytes per
        // 4-column group; every thread then arrives on the peer's barrier,
        // release), then waits for the peer's half, adds it to its own 64
        // columns (fp32 addition of two terms, so both ranks form the same
        // sums), converts into the same staging bytes (each warp has read its
        // region first) and TMA-stores. The staging area is idle until then,
        // so no CTA waits for its peer's MMAs before sending.
        const uint32_t me = u.seg, peer = me ^ 1u;
        if (epi_tid == 0) HG_TR(3);
        uint8_t* stg = staging + (warp - 2) * 8192;
        const uint32_t rbuf = mapa_shared(smem_u32(stg), peer);
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + peer * 64 + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_cluster_v4(rbuf + ((uint32_t(c / 32) * 8u + j) * 32u + lane) * 16u, r[4 * j],
                                 r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        }
        if (epi_tid == 0) HG_TR(5);
        mbar_arrive_cluster(mapa_shared(smem_u32(recv), peer));
        if (!mbar_wait_cluster(recv, 0, abort_flag, p.status, kWdEpilogueTmemFull)) break;
        if (epi_tid == 0) HG_TR(6);
        const float4* r4 = reinterpret_cast<const float4*>(stg);
        {
          const uint32_t c = me * 64;
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(taddr + c, r0);
          tmem_ld_32x32b_x32(taddr + c + 32, r1);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 x0 = r4[j * 32 + lane];
            const float4 x1 = r4[(8 + j) * 32 + lane];
            r0[4 * j] = __float_as_uint(__uint_as_float(r0[4 * j]) + x0.x);
            r0[4 * j + 1] = __float_as_uint(__uint_as_float(r0[4 * j + 1]) + x0.y);
            r0[4 * j + 2] = __float_as_uint(__uint_as_float(r0[4 * j + 2]) + x0.z);
            r0[4 * j + 3] = __float_as_uint(__uint_as_float(r0[4 * j + 3]) + x0.w);
            r1[4 * j] = __float_as_uint(__uint_as_float(r1[4 * j]) + x1.x);
            r1[4 * j + 1] = __float_as_uint(__uint_as_float(r1[4 * j + 1]) + x1.y);
            r1[4 * j + 2] = __float_as_uint(__uint_as_float(r1[4 * j + 2]) + x1.z);
            r1[4 * j + 3] = __float_as_uint(__uint_as_float(r1[4 * j + 3]) + x1.w);
          }
          __syncwarp();  // every lane has read the received partials
          uint8_t* buf = stg;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* src = j < 4 ? &r0[8 * j] : &r1[8 * (j - 4)];
            uint4 v;
            v.x = pack_half2(p.alpha * __uint_as_float(src[0]), p.alpha * __uint_as_float(src[1]));
            v.y = pack_half2(p.alpha * __uint_as_float(src[2]), p.alpha * __uint_as_float(src[3]));
            v.z = pack_half2(p.alpha * __uint_as_float(src[4]), p.alpha * __uint_as_float(src[5]));
            v.w = pack_half2(p.alpha * __uint_as_float(src[6]), p.alpha * __uint_as_float(src[7]));
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((uint32_t(j) ^ (lane & 7u)) * 16)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, buf, int(col0 + c), int(row0 + q * 32));
            bulk_commit_group();
          }
          if (epi_tid == 0) HG_TR(7);
        }
      } else if (!u.partial && p.tma_store) {
        // 64-column chunks: TMEM -> registers -> fp16 -> 128-byte-swizzled
        // smem rows (conflict-free) -> one TMA store of 32 rows x 64 columns
        // per warp. Two staging buffers per warp; TMA clips the ragged edge.
        uint8_t* stg = staging + (warp - 2) * 8192;
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(taddr + c, r0);
          tmem_ld_32x32b_x32(taddr + c + 32, r1);
          tmem_ld_wait();
          uint8_t* buf = stg + ((c / 64) & 1) * 4096;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* src = j < 4 ? &r0[8 * j] : &r1[8 * (j - 4)];
            uint4 v;
            v.x = pack_half2(p.alpha * __uint_as_float(src[0]), p.alpha * __uint_as_float(src[1]));
            v.y = pack_half2(p.alpha * __uint_as_float(src[2]), p.alpha * __uint_as_float(src[3]));
            v.z = pack_half2(p.alpha * __uint_as_float(src[4]), p.alpha * __uint_as_float(src[5]));
            v.w = pack_half2(p.alpha * __uint_as_float(src[6]), p.alpha * __uint_as_float(src[7]));
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((uint32_t(j) ^ (lane & 7u)) * 16)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, buf, int(col0 + c), int(row0 + q * 32));
            bulk_commit_group();
          }
        }
      } else if (!u.partial) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          store_row_chunk(p, row, col0 + c, v);
        }
      } else {
        // Stream-K contribution: publish the fp32 partial, take a ticket.
        float4* slot = reinterpret_cast<float4*>(p.ws_partials) +
                       ((size_t(sc.cta) * 2 + u.seg) * CG + rank) * (BM * BN / 4);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(slot + partial_index(c / 32, j, row_in_tile),
                   make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
        }
        __threadfence();
        named_barrier_sync(1, 128);
        const uint64_t tile_first = uint64_t(u.sk) * sc.KB;
        const uint32_t c_first = sc.cta_of(tile_first);
        const uint32_t c_last = sc.cta_of(tile_first + sc.KB - 1);
        const uint32_t ncontrib = c_last - c_first + 1;
        if (epi_tid == 0) {
          const unsigned old = atomicAdd(&p.ws_counters[u.sk * CG + rank], 1u);
          const uint32_t last = (old == ncontrib - 1) ? 1u : 0u;
          if (last) atomicExch(&p.ws_counters[u.sk * CG + rank], 0u);
          *bcast = last;
        }
        named_barrier_sync(1, 128);
        const bool last = *bcast != 0;
        if (last) {
          __threadfence();
          // Sum the partials in contributor order (deterministic), two
          // 32-column chunks at a time so 16 loads are in flight per thread.
#pragma unroll 1
          for (int c = 0; c < BN; c += 64) {
            float v0[32], v1[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v0[j] = v1[j] = 0.f;
#pragma unroll 1
            for (uint32_t cc = c_first; cc <= c_last; ++cc) {
              const uint32_t seg = (sc.I * cc / sc.Psk) / sc.KB == u.sk ? 0u : 1u;
              const float4* s4 = reinterpret_cast<const float4*>(p.ws_partials) +
                                 ((size_t(cc) * 2 + seg) * CG + rank) * (BM * BN / 4);
              float4 x0[8], x1[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                x0[j] = __ldcg(s4 + partial_index(c / 32, j, row_in_tile));
                x1[j] = __ldcg(s4 + partial_index(c / 32 + 1, j, row_in_tile));
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                v0[4 * j] += x0[j].x; v0[4 * j + 1] += x0[j].y;
                v0[4 * j + 2] += x0[j].z; v0[4 * j + 3] += x0[j].w;
                v1[4 * j] += x1[j].x; v1[4 * j + 1] += x1[j].y;
                v1[4 * j + 2] += x1[j].z; v1[4 * j + 3] += x1[j].w;
              }
              // the partial is dead once summed: drop its L2 lines without a
              // write-back to DRAM (a 128-byte line holds 8 rows of one
              // float4 column; every lane of the warp has its values)
              __syncwarp();
              if ((row_in_tile & 7u) == 0) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  l2_discard_line(s4 + partial_index(c / 32, j, row_in_tile));
                  l2_discard_line(s4 + partial_index(c / 32 + 1, j, row_in_tile));
                }
              }
            }
            store_row_chunk(p, row, col0 + c, v0);
            store_row_chunk(p, row, col0 + c + 32, v1);
          }
        }
        // keep the broadcast slot stable until all threads have read it
        named_barrier_sync(1, 128);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (CG == 2 && rank == 1)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));  // the leader's MMA waits
        else
          mbar_arrive(&tempty[buf]);
      }
      ++i;
    }
    // staging smem must stay valid until the TMA stores have read it
    if (lane == 0) bulk_wait_group<0>();
    if (epi_tid == 0) HG_TR(10);
    __syncwarp();
  }

  tc_fence_before();
  if (CG == 2 || p.ksplit2)
    cluster_sync();  // no CTA exits while its peer may still use its memory
  else
    __syncthreads();
  if (p.dyn && rank == 0 && threadIdx.x == 0) {
    // the last leader CTA to finish puts the tile counter back to zero (every
    // leader has taken its final tile id before it gets here)
    const uint32_t leaders = CG == 2 ? gridDim.x >> 1 : gridDim.x;
    __threadfence();
    if (atomicAdd(p.ws_dyn + 1, 1u) == leaders - 1) {
      atomicExch(p.ws_dyn, 0u);
      atomicExch(p.ws_dyn + 1, 0u);
    }
  }
  if (threadIdx.x == 64) HG_TR(8);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, C_::kTmemCols);
    else
      tmem_dealloc(tmem_base, C_::kTmemCols);
  }
}

}  // namespace hgemm
}  // namespace felix_sm100

#ifdef FELIX_HGEMM_TRACE
extern "C" void hg_trace_fetch(void* dst) {
  cudaMemcpyFromSymbol(dst, felix_sm100::hgemm::g_hg_trace, sizeof(felix_sm100::hgemm::g_hg_trace));
}
extern "C" void hg_tiles_fetch(void* dst) {
  cudaMemcpyFromSymbol(dst, felix_sm100::hgemm::g_hg_tiles, sizeof(felix_sm100::hgemm::g_hg_tiles));
}
#endif

// ============================================================ host launcher
namespace felix_impl {

using namespace felix_sm100::hgemm;

namespace {

template <int BN, int CG = 1, int SUB = (CG == 2 ? 2 : 1)>
int configure_once(int device) {
  static PerDeviceOnce once;
  return once.run(device, [] {
    return int(cudaFuncSetAttribute(felix_sm100::hgemm::hgemm_persistent_kernel<BN, CG, SUB>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg<BN, CG, SUB>::kSmemBytes));
  });
}

struct Plan {
  int bn;
  bool pair;     // CTA pairs: tiles, grid and units counted per pair (grid launched x 2)
  int sub;       // 64-deep k-blocks per stage (2: 32 KB 3-D loads; kblocks count 128-deep)
  bool ksplit2;  // 2-CTA clusters, each tile's K split in halves (grid = 2 x tiles)
  uint32_t tiles_m, tiles_n, kblocks, tiles;
  uint32_t grid;
  uint32_t dp_tiles, sk_tiles;
  uint64_t sk_iters;
};

Plan plan_for(uint32_t M, uint32_t N, uint32_t K, int bn, const HgemmOptions& o, int num_sms) {
  Plan pl{};
  pl.bn = bn;
  pl.sub = 1;
  pl.tiles_m = (M + BM - 1) / BM;
  pl.tiles_n = (N + pl.bn - 1) / pl.bn;
  pl.kblocks = (K + BK - 1) / BK;
  pl.tiles = pl.tiles_m * pl.tiles_n;
  uint32_t P = uint32_t(num_sms);
  if (o.max_ctas > 0 && uint32_t(o.max_ctas) < P) P = uint32_t(o.max_ctas);
  const uint32_t rem = pl.tiles % P;
  bool use_sk;
  if (o.stream_k == 1) {
    use_sk = false;
  } else if (o.stream_k == 2) {
    use_sk = rem != 0 && pl.kblocks >= 2;
  } else {
    // Spread the incomplete wave by k-iterations when it leaves SMs idle and
    // each CTA still gets a useful k-range.
    // Narrow tiles have cheap fix-ups (32 KB partials at BN = 64), so any
    // incomplete wave is worth spreading; wide tiles only when the wave is
    // clearly incomplete.
    const uint32_t pct = bn == 64 ? 100 : 85;
    // Only worth it while whole-tile waves would waste more than ~5% of the
    // SMs: with many waves (e.g. 16384^3: 55 waves, 1.2% loss) the fix-up
    // traffic costs more than the quantisation it removes.
    const uint64_t waves = (pl.tiles + P - 1) / P;
    const bool dp_wasteful = uint64_t(pl.tiles) * 100 < waves * P * 95;
    use_sk = rem != 0 && dp_wasteful && pl.kblocks >= 8 && rem * 100 < P * pct &&
             uint64_t(rem) * pl.kblocks >= uint64_t(P) * 4;
  }
  if (use_sk) {
    pl.sk_tiles = rem;
    pl.dp_tiles = pl.tiles - rem;
    pl.sk_iters = uint64_t(rem) * pl.kblocks;
    pl.grid = P;
  } else {
    pl.sk_tiles = 0;
    pl.dp_tiles = pl.tiles;
    pl.sk_iters = 0;
    pl.grid = pl.tiles < P ? pl.tiles : P;
  }
  return pl;
}

#ifndef FELIX_HGEMM_SK_HALVES
#define FELIX_HGEMM_SK_HALVES 1
#endif
#ifndef FELIX_HGEMM_DYN_WAVES
#define FELIX_HGEMM_DYN_WAVES 4
#endif
// Whole tiles are handed out at run time (TileQueue) when there are at least
// four waves of them; fewer waves do not drift apart enough to matter.
bool uses_dynamic_tiles(const Plan& pl) {
  if (pl.ksplit2) return false;
  return pl.grid > 0 && pl.dp_tiles >= uint32_t(FELIX_HGEMM_DYN_WAVES) * pl.grid;
}

// Library or caller workspace a plan needs: the counter block (stream-K
// tickets, the dynamic tile counter) plus the stream-K partial slots.
size_t workspace_need(const Plan& pl) {
  if (pl.sk_tiles)
    return kWsCounterBytes + size_t(pl.grid) * 2 * (pl.pair ? 2 : 1) * BM * pl.bn * sizeof(float);
  return uses_dynamic_tiles(pl) ? kWsCounterBytes : 0;
}

// Automatic choice of CTA pairs: large enough for at least one wave of
// 256 x 256 tiles, and whole 64-wide k-blocks (and n-chunks for "nn") so that
// the 32 KB 3-D loads are exact. pair_shape_ok carries the layout condition.
bool auto_pair(uint32_t M, uint32_t N, uint32_t K, const HgemmOptions& o, int num_sms,
               bool pair_shape_ok) {
  if (o.cta_pair != 0 || o.block_n != 0 || o.stream_k != 0 || o.max_ctas != 0) return false;
  if (!pair_shape_ok || M < 256 || N < 256 || K < 512 || K % 64 != 0) return false;
  const uint64_t pair_tiles = uint64_t((M + 255) / 256) * ((N + 255) / 256);
  return pair_tiles >= uint64_t(num_sms / 2);
}

Plan make_plan(uint32_t M, uint32_t N, uint32_t K, const HgemmOptions& o, int num_sms,
               bool pair_shape_ok = true) {
  if (o.cta_pair == 2 || auto_pair(M, N, K, o, num_sms, pair_shape_ok)) {
    // 256 x 256 tiles, one unit per CTA pair: plan as 128-row tiles of
    // ceil(M / 2) rows over num_sms / 2 "CTAs"
    HgemmOptions op = o;
    if (op.max_ctas > 0) op.max_ctas = op.max_ctas / 2 > 0 ? op.max_ctas / 2 : 1;
    // (k-blocks of 128 = two 64-deep ones per stage: plan with K / 2)
    Plan pl = plan_for((M + 1) / 2, N, (K + 1) / 2, 256, op, num_sms / 2);
    pl.pair = true;
    return pl;
  }
  if (o.block_n) return plan_for(M, N, K, o.block_n, o, num_sms);
  // Fewer 128x256 tiles than SMs (skinny / decode shapes): the stream-K
  // fix-up of 128 KB partials with many contributors per tile becomes a
  // latency-bound tail, so narrow the tile until there are at least ~0.8
  // tiles per SM (BN = 64 at most halves the A re-reads' efficiency, which
  // only matters when M is large, and then tiles are plentiful).
  const uint32_t tiles_m = (M + BM - 1) / BM;
  int bn = N >= 256 ? 256 : 128;
  while (bn > 128 && uint64_t(tiles_m) * ((N + bn - 1) / bn) * 5 < uint64_t(num_sms) * 4) bn /= 2;
  return plan_for(M, N, K, bn, o, num_sms);
}

}  // namespace

size_t hgemm_workspace_bytes(uint32_t M, uint32_t N, uint32_t K, const HgemmOptions& o,
                             int num_sms) {
  // the larger of the pair and single-CTA plans (the layout is not known here)
  size_t need = 0;
  for (int pair_ok = 0; pair_ok < 2; ++pair_ok) {
    Plan pl = make_plan(M, N, K, o, num_sms, pair_ok != 0);
    const size_t n = workspace_need(pl);
    need = n > need ? n : need;
  }
  return need;
}

FelixCode hgemm_launch(uint32_t M, uint32_t N, uint32_t K, float alpha, const __half* A,
                       const __half* B, float beta, __half* C, bool b_kn, const HgemmOptions& o,
                       void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (M == 0 || N == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  if (!C) return api_error("hgemm: null C");
  if (K == 0) {
    // C = beta * C: a zero-depth product; the tensor-core path needs K > 0.
    return scale_half_matrix(C, size_t(M) * N, beta, stream);
  }
  if (!A || !B) return api_error("hgemm: null pointer");
  if (o.block_n != 0 && o.block_n != 64 && o.block_n != 128 && o.block_n != 256)
    return api_error("hgemm: block_n must be 0, 64, 128 or 256");
  // TMA: global row strides must be multiples of 16 bytes, bases 16-byte aligned.
  if (K % 8 != 0) return api_error("hgemm: K must be a multiple of 8 (16-byte rows for TMA)");
  if (b_kn && N % 8 != 0) return api_error("hgemm nn: N must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15u)
    return api_error("hgemm: A and B must be 16-byte aligned");
  if ((N % 8 == 0) && (reinterpret_cast<uintptr_t>(C) & 15u))
    return api_error("hgemm: C must be 16-byte aligned");

  DeviceInfo* dev = current_device_info();
  if (!dev) return launch_error(cudaGetLastError(), "hgemm: no CUDA device");
  // 3-D views (two 64-wide k-blocks per 32 KB request) are exact only for
  // whole 64-wide blocks: K, and N when B is K x N
  const bool sub2_ok = (K % 64 == 0) && (!b_kn || N % 64 == 0);
  Plan pl = make_plan(M, N, K, o, dev->num_sms, sub2_ok);
  if (pl.pair && !sub2_ok)
    return api_error("hgemm: CTA pairs need K (and N when B is K x N) multiples of 64");
  // Many waves of "nt" pair tiles: 256 x 512 tiles (two N = 256 MMAs per k
  // step, one TMEM accumulator). Per output they read 3/4 of the operand bytes
  // of 256 x 256 tiles; the kernel is power-capped at these sizes, so fewer
  // bytes means a higher clock: 16384^3 5.79 -> 5.59 ms under ncu (DRAM reads
  // 8.9 -> 7.0 GB, 1.30 -> 1.39 GHz), bench 5.67 -> 5.51 ms; 8192^3 697 -> 683 us.
  // 256 x 512 tiles load one 64-deep k-block per stage (48 KB per CTA, four
  // stages) rather than two (96 KB, two stages): 8192^3 676 vs 678 us.
  constexpr int kWideSub = 1;
  bool wide = false;
  {
    const uint64_t wide_tiles = uint64_t((M + 255) / 256) * ((N + 511) / 512);
    if (pl.pair && !b_kn && o.block_n == 0 && o.stream_k == 0 && o.max_ctas == 0 &&
        o.cta_pair == 0 && wide_tiles >= 4u * uint64_t(dev->num_sms / 2)) {
      pl = plan_for((M + 1) / 2, N, kWideSub == 2 ? (K + 1) / 2 : K, 512, o, dev->num_sms / 2);
      pl.pair = true;
      pl.sk_tiles = 0;
      pl.sk_iters = 0;
      pl.dp_tiles = pl.tiles;
      pl.grid = pl.tiles < uint32_t(dev->num_sms / 2) ? pl.tiles : uint32_t(dev->num_sms / 2);
      wide = true;
    }
  }
  // C through TMA when nothing has to be read back (beta == 0) and its rows
  // are 16-byte multiples.
  const bool tma_store = beta == 0.f && (N % 8 == 0) &&
                         (reinterpret_cast<uintptr_t>(C) & 15u) == 0;
  // Few tiles, long K, C through TMA: split each 128 x 128 tile's K over a
  // 2-CTA cluster that reduces through DSMEM, instead of stream-K partials in
  // global memory whose fix-up forms a tail (skinny 128 x 8192 x 16384).
  bool ksplit2 = false;
  {
    const uint32_t t128 = ((M + BM - 1) / BM) * ((N + 127) / 128);
    const uint32_t kb = (K + BK - 1) / BK;
    const uint32_t sms = uint32_t(dev->num_sms);
    if (!pl.pair && o.block_n == 0 && o.stream_k == 0 && o.max_ctas == 0 && tma_store &&
        kb >= 64 && 2 * t128 <= sms && 8 * t128 >= 3 * sms) {
      pl = plan_for(M, N, K, 128, o, dev->num_sms);
      ksplit2 = true;
    }
  }
  // 128-wide single-CTA tiles also take stages of two 64-deep k-blocks (32 KB
  // requests) when the view is exact: plan in 128-deep k-blocks
  if (!pl.pair && pl.bn == 128 && sub2_ok && K >= 128) {
    pl = plan_for(M, N, (K + 1) / 2, 128, o, dev->num_sms);
    pl.sub = 2;
  }
  if (pl.pair) pl.sub = wide ? kWideSub : 2;
  if (ksplit2) {
    pl.ksplit2 = true;
    pl.sk_tiles = 0;
    pl.dp_tiles = pl.tiles;
    pl.sk_iters = 0;
    pl.grid = 2 * pl.tiles;
  }

  CUtensorMap tmA, tmB;
  int rc;
  if (pl.sub == 2) {
    // 3-D views [k-block or n-chunk][rows][64]: one 32 KB request = 128 rows x
    // two 64-wide blocks (a pair's CTA loads half of the tile's B rows).
    rc = encode_tmap_3d_f16(&tmA, A, 64, M, K / 64, uint64_t(K) * 2, 128, 64, BM, 2);
    if (rc) return api_error("hgemm: cuTensorMapEncodeTiled(A) failed");
    rc = b_kn ? encode_tmap_3d_f16(&tmB, B, 64, K, N / 64, uint64_t(N) * 2, 128, 64, 128, 2)
              : encode_tmap_3d_f16(&tmB, B, 64, N, K / 64, uint64_t(K) * 2, 128, 64, 128, 2);
    if (rc) return api_error("hgemm: cuTensorMapEncodeTiled(B) failed");
  } else {
    rc = encode_tmap_2d_f16_swizzle(&tmA, A, K, M, uint64_t(K) * 2, BK, BM, kSwizzleK);
    if (rc) return api_error("hgemm: cuTensorMapEncodeTiled(A) failed");
    if (b_kn)
      rc = encode_tmap_2d_f16(&tmB, B, N, K, uint64_t(N) * 2, 64, BK);
    else
      rc = encode_tmap_2d_f16_swizzle(&tmB, B, K, N, uint64_t(K) * 2, BK,
                                      wide ? 128 : pl.bn, kSwizzleK);
    if (rc) return api_error("hgemm: cuTensorMapEncodeTiled(B) failed");
  }
  CUtensorMap tmC;
  if (tma_store && encode_tmap_2d_f16(&tmC, C, N, M, uint64_t(N) * 2, 64, 32))
    return api_error("hgemm: cuTensorMapEncodeTiled(C) failed");
  if (!tma_store) tmC = tmA;  // unused placeholder

  Params p{};
  p.tma_store = tma_store ? 1u : 0u;
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.C = C;
  p.b_mn_major = b_kn ? 1u : 0u;
  p.tiles_m = pl.tiles_m;
  p.tiles_n = pl.tiles_n;
  p.kblocks = pl.kblocks;
  p.dp_tiles = pl.dp_tiles;
  p.sk_tiles = pl.sk_tiles;
  p.sk_iters = pl.sk_iters;
  // Stream-K tail in equal shares: with c = units / sk_tiles >= 2 and K
  // splitting evenly into c parts, c x sk_tiles units take exactly 1/c of a
  // split tile each (the others only whole tiles), so no unit runs two
  // partial units and every split tile has c contributors. Spreading the
  // iterations over all units instead gives some units a second, tiny
  // partial unit and, as the last contributor, its fix-up: 4096^3 with CTA
  // pairs (34 split tiles over 74 pairs, c = 2) 98.3 -> 94.2 us.
  p.sk_units = 0;
  // (not for 512-wide pair tiles, whose single accumulator serialises a
  // unit's epilogue with the next unit: 2048 x 16384 x 16384 707.6 -> 773 us)
  if (FELIX_HGEMM_SK_HALVES && pl.sk_tiles && !wide) {
    const uint32_t units = pl.grid;  // CTAs, or pairs of CTAs
    uint32_t c = units / pl.sk_tiles;
    while (c >= 2 && (pl.kblocks % c != 0 || pl.kblocks / c < 4)) --c;
    if (c >= 2) p.sk_units = c * pl.sk_tiles;
  }
  // Grouped raster height (tiles): the CTAs running at the same time cover a
  // group_m x (CTAs / group_m) block of tiles and share its A and B panels in
  // L2. Measured at 16384^3 with CTA pairs (74 concurrent 256 x 256 tiles):
  // group 2 / 4 / 8 / 16 / 32 read 19.2 / 11.4 / 9.2 / 16.8 / 32.5 GB from
  // DRAM for 1.07 GB of operands, and 8 ran 12 % faster than 16 (the kernel is
  // power-capped there: fewer DRAM bytes, higher clock); 8192^3: 707 vs 718 us.
  // Single-CTA 128 x 256 tiles (148 concurrent): 16 (8192^3: 763 vs 789 us).
  // 256 x 512 pair tiles (four 48 KB stages): 12. DRAM reads at 16384^3 for
  // group 6 / 8 / 10 / 12 / 16 / 20 / 24 / 32: 9.2 / 8.5 / 8.6 / 8.3 / 10.4 /
  // 12.0 / 13.3 / 16.3 GB; 12 and 8 ran fastest (5.49-5.67 ms median).
  p.group_m = wide ? 12u : (pl.pair ? 8u : 16u);
  p.status = dev->status_word;
  p.ksplit2 = pl.ksplit2 ? 1u : 0u;
  p.pair = pl.pair ? 1u : 0u;
  p.dyn = uses_dynamic_tiles(pl) ? 1u : 0u;
  if (pl.sk_tiles || p.dyn) {
    if (uint64_t(pl.sk_tiles) * (pl.pair ? 2 : 1) > kWsMaxCounters - 2)
      return api_error("hgemm: too many stream-K tiles");
    const size_t need = workspace_need(pl);
    if (!workspace) {
      workspace = library_workspace(dev, stream, need);
      if (!workspace) return launch_error(cudaErrorMemoryAllocation, "hgemm: workspace");
    } else if (ws_bytes < need) {
      return api_error("hgemm: workspace too small");
    }
    p.ws_counters = static_cast<unsigned*>(workspace);
    p.ws_dyn = p.ws_counters + (kWsMaxCounters - 2);
    p.ws_partials =
        reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsCounterBytes);
  }

  cudaError_t e;
  if (pl.pair) {
    if ((rc = wide ? configure_once<512, 2, kWideSub>(dev->ordinal)
                   : configure_once<256, 2>(dev->ordinal)))
      return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = wide ? Cfg<512, 2, kWideSub>::kSmemBytes : Cfg<256, 2>::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = wide ? cudaLaunchKernelEx(&cfg, hgemm_persistent_kernel<512, 2, kWideSub>, tmA, tmB, tmC, p)
             : cudaLaunchKernelEx(&cfg, hgemm_persistent_kernel<256, 2>, tmA, tmB, tmC, p);
    if (e != cudaSuccess) return launch_error(e, "hgemm: CTA-pair launch failed");
    return FelixCode{FELIX_SUCCESS, cudaSuccess};
  }
  switch (pl.bn) {
    case 256:
      if ((rc = configure_once<256>(dev->ordinal)))
        return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
      hgemm_persistent_kernel<256>
          <<<pl.grid, kThreads, Cfg<256>::kSmemBytes, stream>>>(tmA, tmB, tmC, p);
      break;
    case 128: {
      // launch the 128-wide kernel with one or two k-blocks per stage, as a
      // 2-CTA cluster for the cluster split-K plan
      auto launch128 = [&](auto kernel, int smem) -> cudaError_t {
        if (!pl.ksplit2) {
          kernel<<<pl.grid, kThreads, smem, stream>>>(tmA, tmB, tmC, p);
          return cudaGetLastError();
        }
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(pl.grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, tmC, p);
      };
      if (pl.sub == 2) {
        if ((rc = configure_once<128, 1, 2>(dev->ordinal)))
          return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
        e = launch128(hgemm_persistent_kernel<128, 1, 2>, Cfg<128, 1, 2>::kSmemBytes);
      } else {
        if ((rc = configure_once<128>(dev->ordinal)))
          return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
        e = launch128(hgemm_persistent_kernel<128>, Cfg<128>::kSmemBytes);
      }
      if (e != cudaSuccess) return launch_error(e, "hgemm: launch failed");
      break;
    }
    default:
      if ((rc = configure_once<64>(dev->ordinal)))
        return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
      hgemm_persistent_kernel<64>
          <<<pl.grid, kThreads, Cfg<64>::kSmemBytes, stream>>>(tmA, tmB, tmC, p);
      break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return launch_error(e, "hgemm: launch failed");
  return FelixCode{FELIX_SUCCESS, cudaSuccess};
}

}  // namespace felix_impl
