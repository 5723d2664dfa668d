// k-th value selection per slice (top-k radix select) for sm_100a.
// out[s] = the k-th largest (largest != 0) or k-th smallest value of
// data[s * slice_size .. (s + 1) * slice_size), fp32.
// Replaces felix::sorting_radix_select_launch / "sorting_radix_select"
// (reference: include/felix/felix.hpp:17-20,
// src/felix/topk/sorting_radix_select_kernel_launch.cu:7-38,
// kernels/sorting_radix_select.cuh:153-213), with the same ordering: floats are
// mapped to order-preserving uint32 keys (negative values bit-inverted, others
// with the sign bit set; NaN compares above +inf), and the key found maps back
// to the exact value bits (so -0.0 and +0.0 are distinct, -0.0 < +0.0).
//
// Design (HBM-bound integer work, no tensor cores):
//   * the k-th largest is the (n - k)-th smallest (0-based rank), so one
//     ascending select serves both directions;
//   * radix passes, most significant digit first; each pass builds a
//     histogram of the keys that still match the chosen prefix and picks the
//     digit where the running count passes the rank;
//   * many slices: one CTA per slice; slices up to 48K values are staged once
//     into shared memory (so HBM is read once). Aligned staged slices take
//     three passes (11-, 11- and 10-bit digits), the third over a compacted
//     list of candidates only; the others four 8-bit passes with per-warp
//     sub-histograms against atomic contention;
//   * few large slices: every pass is a grid-wide histogram kernel over all
//     SMs plus a one-warp digit pick per slice, with the histograms and the
//     per-slice (prefix, rank) state in library scratch.
#include <cuda_runtime.h>
#include <cstdint>
#include <type_traits>

#include "felix_internal.h"
#include "sm100_ptx.cuh"

namespace felix_sm100 {
namespace topk {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kSmemKeys = 48 * 1024;  // staged keys per slice (192 KB)
constexpr uint32_t kChunkBytes = 16 * 1024;  // bulk copies of a staged slice
constexpr uint32_t kChunks = kSmemKeys * 4 / kChunkBytes;

__device__ __forceinline__ uint32_t to_key(float v) {
  const uint32_t x = __float_as_uint(v);
  if (v != v) return 0xffffffffu;  // NaN above everything
  return x ^ ((x & 0x80000000u) ? 0xffffffffu : 0x80000000u);
}
// The same map on the value's bits, integer operations only.
__device__ __forceinline__ uint32_t to_key_bits(uint32_t x) {
  const uint32_t k = x ^ (uint32_t(int32_t(x) >> 31) | 0x80000000u);
  return (x & 0x7fffffffu) > 0x7f800000u ? 0xffffffffu : k;  // NaN above everything
}
__device__ __forceinline__ float from_key(uint32_t k) {
  return __uint_as_float(k ^ ((k & 0x80000000u) ? 0x80000000u : 0xffffffffu));
}

// Digit whose cumulative count first exceeds `rank` (counts of one pass), and
// the count of keys below it. Executed by one full warp.
__device__ __forceinline__ void pick_digit(const uint32_t* hist, uint32_t rank, uint32_t& digit,
                                          uint32_t& below) {
  const uint32_t lane = threadIdx.x & 31u;
  uint32_t c[8], sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = hist[lane * 8 + i];
    sum += c[i];
  }
  // exclusive prefix of the 32 lane sums
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= uint32_t(o)) incl += v;
  }
  const uint32_t excl = incl - sum;
  const bool mine = rank >= excl && rank < incl;
  const uint32_t who = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
  uint32_t d = 0, b = 0;
  if (lane == who) {
    uint32_t run = excl;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (rank < run + c[i]) {
        d = lane * 8 + i;
        b = run;
        break;
      }
      run += c[i];
    }
  }
  digit = __shfl_sync(0xffffffffu, d, who);
  below = __shfl_sync(0xffffffffu, b, who);
}

// One CTA per slice.
__global__ void __launch_bounds__(kThreads) select_per_slice_kernel(const float* __restrict__ data,
                                                                  float* __restrict__ out,
                                                                  uint32_t slice_size, uint32_t k,
                                                                  int largest, int staged,
                                                                  unsigned* status) {
  extern __shared__ __align__(16) uint32_t keys[];    // [slice_size] when staged
  __shared__ uint32_t hist[kWarps][256];
  __shared__ uint32_t merged[256];
  __shared__ uint32_t s_prefix, s_rank;
  __shared__ __align__(8) uint64_t chunk_full[kChunks];
  __shared__ int s_abort;
  const uint32_t t = threadIdx.x, w = t / 32;
  const float* src = data + size_t(blockIdx.x) * slice_size;
  // sub-histograms: one per warp for large slices, fewer for small ones (each
  // pass clears and merges them all)
  const uint32_t nh = slice_size >= 16384 ? uint32_t(kWarps) : slice_size >= 4096 ? 4u : 1u;
  uint32_t* my_hist = hist[w % nh];
  // Staged and 16-byte aligned: the slice streams into shared memory as bulk
  // copies of kChunkBytes, each completing on its own mbarrier, and the first
  // pass converts and counts each chunk as soon as it lands (HBM read once,
  // the load overlapped with the first histogram).
  const bool bulk = staged && (slice_size & 3u) == 0 &&
                    (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  const uint32_t bytes = slice_size * 4u;
  const uint32_t nchunks = bulk ? (bytes + kChunkBytes - 1) / kChunkBytes : 0u;
  if (t == 0) {
    s_prefix = 0;
    s_rank = largest ? slice_size - k : k - 1;
    s_abort = 0;
    for (uint32_t c = 0; c < nchunks; ++c) felix_sm100::mbar_init(&chunk_full[c], 1);
    felix_sm100::fence_mbar_init();
  }
  for (uint32_t i = t; i < nh * 256; i += kThreads) (&hist[0][0])[i] = 0;
  __syncthreads();
  if (bulk) {
    if (t == 0) {
      for (uint32_t c = 0; c < nchunks; ++c) {
        const uint32_t off = c * kChunkBytes;
        const uint32_t len = bytes - off < kChunkBytes ? bytes - off : kChunkBytes;
        felix_sm100::mbar_arrive_expect_tx(&chunk_full[c], len);
        felix_sm100::bulk_load_1d(reinterpret_cast<uint8_t*>(keys) + off,
                                  reinterpret_cast<const uint8_t*>(src) + off, len, &chunk_full[c]);
      }
    }
    // pass 1 (top digit, every key counts) chunk by chunk as the copies land
    bool ok = true;
    for (uint32_t c = 0; c < nchunks; ++c) {
      if (ok && !felix_sm100::mbar_wait(&chunk_full[c], 0, &s_abort, status,
                                       felix_sm100::kWdTopkLoad))
        ok = false;
      const uint32_t beg = c * (kChunkBytes / 4);
      const uint32_t end = min(slice_size, beg + kChunkBytes / 4);
      if (ok) {
        // 16-byte pieces (the chunk bounds are multiples of 4 keys here)
        uint4* k4 = reinterpret_cast<uint4*>(keys);
        for (uint32_t i = beg / 4 + t; i < end / 4; i += kThreads) {
          uint4 v = k4[i];
          v.x = to_key(__uint_as_float(v.x));
          v.y = to_key(__uint_as_float(v.y));
          v.z = to_key(__uint_as_float(v.z));
          v.w = to_key(__uint_as_float(v.w));
          k4[i] = v;
          atomicAdd(&my_hist[v.x >> 24], 1u);
          atomicAdd(&my_hist[v.y >> 24], 1u);
          atomicAdd(&my_hist[v.z >> 24], 1u);
          atomicAdd(&my_hist[v.w >> 24], 1u);
        }
      }
    }
    ok = __syncthreads_and(ok) != 0;  // one decision for the whole CTA
    if (!ok) {
      // a copy never landed (watchdog recorded): wait (bounded) for the rest
      // so that none is in flight when the CTA exits
      if (t == 0) {
        int dummy = 0;
        for (uint32_t c = 0; c < nchunks; ++c)
          felix_sm100::mbar_wait(&chunk_full[c], 0, &dummy, status, felix_sm100::kWdDrain,
                                 100000000ull);
      }
      __syncthreads();
      return;
    }
  } else if (staged) {
    for (uint32_t i = t; i < slice_size; i += kThreads) keys[i] = to_key(__ldg(src + i));
  }
  uint32_t mask = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (pass > 0 || !bulk) {
      if (pass > 0) {
        for (uint32_t i = t; i < nh * 256; i += kThreads) (&hist[0][0])[i] = 0;
      }
      __syncthreads();
      const uint32_t prefix = s_prefix;
      if (bulk) {
        // staged keys, 4 per 16-byte read
        const uint4* k4 = reinterpret_cast<const uint4*>(keys);
        for (uint32_t i = t; i < slice_size / 4; i += kThreads) {
          const uint4 v = k4[i];
          if ((v.x & mask) == prefix) atomicAdd(&my_hist[(v.x >> shift) & 255u], 1u);
          if ((v.y & mask) == prefix) atomicAdd(&my_hist[(v.y >> shift) & 255u], 1u);
          if ((v.z & mask) == prefix) atomicAdd(&my_hist[(v.z >> shift) & 255u], 1u);
          if ((v.w & mask) == prefix) atomicAdd(&my_hist[(v.w >> shift) & 255u], 1u);
        }
      } else {
        for (uint32_t i = t; i < slice_size; i += kThreads) {
          const uint32_t key = staged ? keys[i] : to_key(__ldg(src + i));
          if ((key & mask) == prefix) atomicAdd(&my_hist[(key >> shift) & 255u], 1u);
        }
      }
    }
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (uint32_t b = t; b < 256; b += kThreads) {
      uint32_t s = 0;
      for (uint32_t ww = 0; ww < nh; ++ww) s += hist[ww][b];
      merged[b] = s;
    }
    __syncthreads();
    if (w == 0) {
      uint32_t d, below;
      pick_digit(merged, s_rank, d, below);
      if (t == 0) {
        s_rank -= below;
        s_prefix = prefix | (d << shift);
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  if (t == 0) out[blockIdx.x] = from_key(s_prefix);
}

// Staged slices that are 16-byte aligned (n % 4 == 0): three passes over
// 11-, 11- and 10-bit digits instead of four over 8-bit ones, and only the
// first two over the whole slice. Pass 1 converts and counts the top 11 bits
// of each bulk-copied chunk as it lands; pass 2 reads the staged keys once
// more, counts the next 11 bits of the keys whose top digit matches and
// appends those keys to a candidate list behind the slice in shared memory
// (each warp its own region, positions from ballots: no atomics); pass 3
// counts the last 10 bits over the candidates only, or over the staged keys
// again when the list overflowed (many equal top digits). Digits are picked
// by the whole CTA (a block-wide scan of the 2048 counts).
#ifdef FELIX_TOPK_TRACE
// Development-only per-CTA timeline (compiled out of the library build).
__device__ unsigned long long g_tk_trace[8192][8];
#define TK_TR(ev)                                                             \
  do {                                                                        \
    if (threadIdx.x == 0 && blockIdx.x < 8192)                                \
      g_tk_trace[blockIdx.x][ev] = felix_sm100::globaltimer_ns();             \
  } while (0)
#else
#define TK_TR(ev) \
  do {            \
  } while (0)
#endif
constexpr uint32_t kBins = 2048;
constexpr uint32_t kL2MinKeys = 8192;  // unstaged three-pass select from this slice size
constexpr uint32_t kSubH = 2;  // sub-histograms (warp w counts into w % kSubH)
// dynamic shared memory of the staged kernel: the slice plus the candidates
// (with the static part, 16.2 KB, within the 227 KB per-CTA limit)
constexpr uint32_t kStagedDynBytes = 210 * 1024;

// Digit whose cumulative count first exceeds `rank` among nbins counts (a
// multiple of kThreads, at most 4 per thread); called by every thread of the
// CTA. s_out[0] = the digit, s_out[1] = the count of keys below it, both
// visible to every thread on return.
__device__ __forceinline__ void pick_digit_cta(const uint32_t* h, uint32_t nbins, uint32_t rank,
                                               uint32_t* wsum, uint32_t* s_out) {
  const uint32_t t = threadIdx.x, lane = t & 31u, w = t >> 5;
  const uint32_t per = nbins / kThreads;
  uint32_t c[4], sum = 0;
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) {
    c[i] = i < per ? h[t * per + i] : 0u;
    sum += c[i];
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= uint32_t(o)) incl += v;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  uint32_t off = 0;
  for (uint32_t ww = 0; ww < w; ++ww) off += wsum[ww];
  const uint32_t excl = off + incl - sum;
  if (rank >= excl && rank < excl + sum) {
    uint32_t run = excl;
    for (uint32_t i = 0; i < per; ++i) {
      if (rank < run + c[i]) {
        s_out[0] = t * per + i;
        s_out[1] = run;
        break;
      }
      run += c[i];
    }
  }
  __syncthreads();
}

// STAGED = false: the same three passes without staging. Pass 1 streams the
// slice from HBM, passes 2 (and 3 when the candidates overflow) read it again
// through the L2, which still holds it: shared memory then holds only the
// histograms and the candidates, so several CTAs share an SM and their loads
// overlap each other's passes.
template <bool STAGED>
__global__ void __launch_bounds__(kThreads, 4) select_radix3_kernel(const float* __restrict__ data,
                                                                 float* __restrict__ out,
                                                                 uint32_t slice_size, uint32_t k,
                                                                 int largest, uint32_t cap,
                                                                 unsigned* status) {
  // staged: [slice_size] keys, then [cap] candidates; otherwise the candidates
  extern __shared__ __align__(16) uint32_t dyn[];
  __shared__ uint32_t hist[kSubH][kBins];
  __shared__ uint32_t wsum[kWarps], s_pick[2], s_wcount[kWarps];
  __shared__ __align__(8) uint64_t chunk_full[kChunks];
  __shared__ int s_abort;
  const uint32_t t = threadIdx.x, w = t / 32, lane = t % 32;
  uint32_t* keys = dyn;
  uint32_t* cand = STAGED ? dyn + slice_size : dyn;
  uint32_t* my_hist = hist[w % kSubH];
  const float* src = data + size_t(blockIdx.x) * slice_size;
  const uint32_t bytes = slice_size * 4u;
  const uint32_t nchunks = STAGED ? (bytes + kChunkBytes - 1) / kChunkBytes : 0u;
  const uint4* g4 = reinterpret_cast<const uint4*>(src);
  uint4* k4 = reinterpret_cast<uint4*>(keys);
  const uint32_t n4 = slice_size / 4;
  // four keys of 16-byte group i (converted)
  auto load4 = [&](uint32_t i) -> uint4 {
    if constexpr (STAGED) {
      return k4[i];
    } else {
      uint4 v = __ldcg(g4 + i);
      v.x = to_key_bits(v.x);
      v.y = to_key_bits(v.y);
      v.z = to_key_bits(v.z);
      v.w = to_key_bits(v.w);
      return v;
    }
  };
  auto clear_hist = [&]() {
    for (uint32_t i = t; i < kSubH * kBins; i += kThreads) (&hist[0][0])[i] = 0;
  };
  auto merge_hist = [&](uint32_t nbins) {
    for (uint32_t b = t; b < nbins; b += kThreads) {
      uint32_t v = hist[0][b];
#pragma unroll
      for (uint32_t h = 1; h < kSubH; ++h) v += hist[h][b];
      hist[0][b] = v;
    }
  };
  TK_TR(0);
  if (t == 0) {
    s_abort = 0;
    for (uint32_t c = 0; c < nchunks; ++c) felix_sm100::mbar_init(&chunk_full[c], 1);
    felix_sm100::fence_mbar_init();
  }
  clear_hist();
  __syncthreads();
  if (t == 0) {
    for (uint32_t c = 0; c < nchunks; ++c) {
      const uint32_t off = c * kChunkBytes;
      const uint32_t len = bytes - off < kChunkBytes ? bytes - off : kChunkBytes;
      felix_sm100::mbar_arrive_expect_tx(&chunk_full[c], len);
      felix_sm100::bulk_load_1d(reinterpret_cast<uint8_t*>(keys) + off,
                                reinterpret_cast<const uint8_t*>(src) + off, len, &chunk_full[c]);
    }
  }
  // pass 1: convert each chunk in place as it lands and count the top 11 bits
  // (unstaged: stream the slice, four 16-byte loads in flight per thread)
  bool ok = true;
  if constexpr (!STAGED) {
    for (uint32_t i0 = t; i0 < n4; i0 += 4 * kThreads) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t i = i0 + u * kThreads;
        if (i < n4) v[u] = __ldcg(g4 + i);
      }
      // counted by the raw bits 31..21 (a permutation of the key digit,
      // undone when the sub-histograms merge); every NaN goes to raw digit
      // 1023, which holds only NaNs and maps to key digit 2047, where the
      // key of every NaN lies
      auto raw_bin = [](uint32_t x) -> uint32_t {
        return (x & 0x7fffffffu) > 0x7f800000u ? 1023u : x >> 21;
      };
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + u * kThreads < n4) {
          atomicAdd(&my_hist[raw_bin(v[u].x)], 1u);
          atomicAdd(&my_hist[raw_bin(v[u].y)], 1u);
          atomicAdd(&my_hist[raw_bin(v[u].z)], 1u);
          atomicAdd(&my_hist[raw_bin(v[u].w)], 1u);
        }
      }
    }
  }
  for (uint32_t c = 0; c < nchunks; ++c) {
    if (ok && !felix_sm100::mbar_wait(&chunk_full[c], 0, &s_abort, status,
                                     felix_sm100::kWdTopkLoad))
      ok = false;
    const uint32_t beg = c * (kChunkBytes / 16);
    const uint32_t end = min(slice_size / 4, beg + kChunkBytes / 16);
    if (ok) {
      for (uint32_t i = beg + t; i < end; i += kThreads) {
        uint4 v = k4[i];
        v.x = to_key_bits(v.x);
        v.y = to_key_bits(v.y);
        v.z = to_key_bits(v.z);
        v.w = to_key_bits(v.w);
        k4[i] = v;
        atomicAdd(&my_hist[v.x >> 21], 1u);
        atomicAdd(&my_hist[v.y >> 21], 1u);
        atomicAdd(&my_hist[v.z >> 21], 1u);
        atomicAdd(&my_hist[v.w >> 21], 1u);
      }
    }
  }
  ok = __syncthreads_and(ok) != 0;
  if (!ok) {
    // a copy never landed (watchdog recorded): wait (bounded) for the rest so
    // that none is in flight when the CTA exits
    if (t == 0) {
      int dummy = 0;
      for (uint32_t c = 0; c < nchunks; ++c)
        felix_sm100::mbar_wait(&chunk_full[c], 0, &dummy, status, felix_sm100::kWdDrain,
                               100000000ull);
    }
    __syncthreads();
    return;
  }
  TK_TR(1);
  if constexpr (STAGED) {
    merge_hist(kBins);
  } else {
    // merge, and move raw digit r to its key digit: r ^ 1024 for the
    // positive half, ~r for the negative one
    uint32_t sums[kBins / kThreads];
#pragma unroll
    for (uint32_t q = 0; q < kBins / kThreads; ++q) {
      const uint32_t b = t + q * kThreads;
      uint32_t v = hist[0][b];
#pragma unroll
      for (uint32_t h = 1; h < kSubH; ++h) v += hist[h][b];
      sums[q] = v;
    }
    __syncthreads();
#pragma unroll
    for (uint32_t q = 0; q < kBins / kThreads; ++q) {
      const uint32_t r = t + q * kThreads;
      hist[0][r < 1024u ? r ^ 1024u : ~r & (kBins - 1)] = sums[q];
    }
  }
  __syncthreads();
  uint32_t rank = largest ? slice_size - k : k - 1;
  pick_digit_cta(hist[0], kBins, rank, wsum, s_pick);
  const uint32_t d1 = s_pick[0];
  rank -= s_pick[1];
  clear_hist();
  __syncthreads();
  TK_TR(2);
  // pass 2: count bits 20..10 of the keys with top digit d1 and collect them,
  // warp w into cand[w * region ..), positions from ballots
  const uint32_t n4w = (n4 + 31u) & ~31u;  // whole warps take part in the ballots
  const uint32_t region = cap / kWarps;
  uint32_t* my_cand = cand + w * region;
  const uint32_t lt = (1u << lane) - 1u;
  uint32_t wn = 0;  // candidates of this warp so far (same in every lane)
  // U 16-byte groups per thread and step, loaded before any candidate is
  // stored (the stores could otherwise alias the loads and serialise them);
  // U = 4 for long slices, 1 for short ones (fewer idle ballots)
  // Unstaged, the match test runs on the raw bits: keys with top digit d1
  // are exactly the values whose bits 31..21 equal t1 (d1 ^ 1024 for the
  // positive half, ~d1 for the negative one), except that NaN bit patterns
  // share the digits 0..3 and 2044..2047 with real values (all NaNs have the
  // key 0xffffffff); for those d1 every key is converted first.
  const bool raw_ok = !STAGED && d1 >= 4u && d1 <= 2043u;
  const uint32_t t1 = d1 >= 1024u ? (d1 ^ 1024u) : (~d1 & 2047u);
  auto compact = [&](auto unroll) {
    constexpr int U = decltype(unroll)::value;
    for (uint32_t i0 = t; i0 < n4w; i0 += U * kThreads) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = i0 + u * kThreads;
        if constexpr (STAGED)
          v[u] = i < n4 ? k4[i] : make_uint4(0u, 0u, 0u, 0u);
        else
          v[u] = i < n4 ? __ldcg(g4 + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = i0 + u * kThreads;
        uint32_t kk[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (!STAGED && !raw_ok) {
#pragma unroll
          for (int j = 0; j < 4; ++j) kk[j] = to_key_bits(kk[j]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool match =
              i < n4 && (raw_ok ? (kk[j] >> 21) == t1 : (kk[j] >> 21) == d1);
          const uint32_t b = __ballot_sync(0xffffffffu, match);
          if (match) {
            const uint32_t key = raw_ok ? to_key_bits(kk[j]) : kk[j];
            atomicAdd(&my_hist[(key >> 10) & (kBins - 1)], 1u);
            const uint32_t pos = wn + __popc(b & lt);
            if (pos < region) my_cand[pos] = key;
          }
          wn += __popc(b);
        }
      }
    }
  };
  if (n4 >= 8 * kThreads)
    compact(std::integral_constant<int, 4>{});
  else
    compact(std::integral_constant<int, 1>{});
  if (lane == 0) s_wcount[w] = wn;
  __syncthreads();
  TK_TR(3);
  merge_hist(kBins);
  __syncthreads();
  pick_digit_cta(hist[0], kBins, rank, wsum, s_pick);
  const uint32_t prefix22 = (d1 << 11) | s_pick[0];
  rank -= s_pick[1];
  clear_hist();
  __syncthreads();
  // pass 3: the last 10 bits of the keys whose top 22 bits match
  bool fits = true;
  for (uint32_t ww = 0; ww < kWarps; ++ww) fits = fits && s_wcount[ww] <= region;
  if (fits) {
    // each warp its own region
    for (uint32_t i = lane; i < wn; i += 32) {
      const uint32_t key = my_cand[i];
      if ((key >> 10) == prefix22) atomicAdd(&my_hist[key & 1023u], 1u);
    }
  } else {
    for (uint32_t i = t; i < n4; i += kThreads) {
      const uint4 v = load4(i);
      if ((v.x >> 10) == prefix22) atomicAdd(&my_hist[v.x & 1023u], 1u);
      if ((v.y >> 10) == prefix22) atomicAdd(&my_hist[v.y & 1023u], 1u);
      if ((v.z >> 10) == prefix22) atomicAdd(&my_hist[v.z & 1023u], 1u);
      if ((v.w >> 10) == prefix22) atomicAdd(&my_hist[v.w & 1023u], 1u);
    }
  }
  __syncthreads();
  merge_hist(1024);
  __syncthreads();
  pick_digit_cta(hist[0], 1024, rank, wsum, s_pick);
  if (t == 0) out[blockIdx.x] = from_key((prefix22 << 10) | s_pick[0]);
  TK_TR(4);
}

// Small slices (<= kWarpKeys values): one warp per slice, the keys held in
// registers (kWarpKeys / 32 per lane), a 256-bin histogram per warp in shared
// memory and warp-level synchronisation only, so a CTA of kWarps warps selects
// kWarps slices at once.
constexpr uint32_t kWarpKeys = 2048;
constexpr int kPerLane = kWarpKeys / 32;

__global__ void __launch_bounds__(kThreads) select_warp_per_slice_kernel(
    const float* __restrict__ data, float* __restrict__ out, uint32_t num_slices,
    uint32_t slice_size, uint32_t k, int largest) {
  __shared__ uint32_t hist[kWarps][256];
  const uint32_t lane = threadIdx.x & 31u, w = threadIdx.x / 32;
  const uint32_t slice = blockIdx.x * kWarps + w;
  if (slice >= num_slices) return;  // whole warps only: no CTA-wide barrier below
  const float* src = data + size_t(slice) * slice_size;
  uint32_t key[kPerLane];
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) {
    const uint32_t i = uint32_t(j) * 32 + lane;  // coalesced across the warp
    key[j] = i < slice_size ? to_key(__ldg(src + i)) : 0u;
  }
  uint32_t* h = hist[w];
  uint32_t prefix = 0, mask = 0;
  uint32_t rank = largest ? slice_size - k : k - 1;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
#pragma unroll
    for (int b = 0; b < 8; ++b) h[lane * 8 + b] = 0;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const uint32_t i = uint32_t(j) * 32 + lane;
      if (i < slice_size && (key[j] & mask) == prefix) atomicAdd(&h[(key[j] >> shift) & 255u], 1u);
    }
    __syncwarp();
    uint32_t d, below;
    pick_digit(h, rank, d, below);
    rank -= below;
    prefix |= d << shift;
    mask |= 255u << shift;
    __syncwarp();
  }
  if (lane == 0) out[slice] = from_key(prefix);
}

// Grid-wide pass for few large slices: histogram of the digit at `shift` of
// the keys of slice blockIdx.y that match state.prefix under `mask`.
struct SliceState {
  uint32_t prefix;
  uint32_t rank;
};

__global__ void __launch_bounds__(kThreads) histogram_pass_kernel(const float* __restrict__ data,
                                                                  uint32_t slice_size, int shift,
                                                                  uint32_t mask,
                                                                  const SliceState* state,
                                                                  uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[kWarps][256];
  const uint32_t t = threadIdx.x, w = t / 32;
  for (uint32_t i = t; i < kWarps * 256; i += kThreads) (&h[0][0])[i] = 0;
  __syncthreads();
  const uint32_t slice = blockIdx.y;
  const uint32_t prefix = state[slice].prefix;
  const float* src = data + size_t(slice) * slice_size;
  const uint32_t n4 = (slice_size & 3u) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0
                          ? slice_size / 4
                          : 0;
  const uint32_t stride = gridDim.x * kThreads;
  for (uint32_t i = blockIdx.x * kThreads + t; i < n4; i += stride) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(src) + i);
    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t key = to_key(vv[j]);
      if ((key & mask) == prefix) atomicAdd(&h[w][(key >> shift) & 255u], 1u);
    }
  }
  for (uint32_t i = n4 * 4 + blockIdx.x * kThreads + t; i < slice_size; i += stride) {
    const uint32_t key = to_key(__ldg(src + i));
    if ((key & mask) == prefix) atomicAdd(&h[w][(key >> shift) & 255u], 1u);
  }
  __syncthreads();
  for (uint32_t b = t; b < 256; b += kThreads) {
    uint32_t s = 0;
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww) s += h[ww][b];
    if (s) atomicAdd(&hist[size_t(slice) * 256 + b], s);
  }
}

// One warp per slice: choose the digit, update (prefix, rank), clear the
// histogram for the next pass; after the last pass write the value.
__global__ void pick_pass_kernel(uint32_t* hist, SliceState* state, int shift, int last,
                                 float* out) {
  const uint32_t slice = blockIdx.x;
  uint32_t* hs = hist + size_t(slice) * 256;
  uint32_t d, below;
  pick_digit(hs, state[slice].rank, d, below);
  __syncwarp();
  for (uint32_t b = threadIdx.x; b < 256; b += 32) hs[b] = 0;
  if (threadIdx.x == 0) {
    state[slice].rank -= below;
    state[slice].prefix |= d << shift;
    if (last) out[slice] = from_key(state[slice].prefix);
  }
}

__global__ void init_state_kernel(SliceState* state, uint32_t num_slices, uint32_t slice_size,
                                  uint32_t k, int largest) {
  const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < num_slices) {
    state[s].prefix = 0;
    state[s].rank = largest ? slice_size - k : k - 1;
  }
}

}  // namespace topk
}  // namespace felix_sm100

#ifdef FELIX_TOPK_TRACE
extern "C" void tk_trace_fetch(void* dst) {
  cudaMemcpyFromSymbol(dst, felix_sm100::topk::g_tk_trace, sizeof(felix_sm100::topk::g_tk_trace));
}
#endif

namespace felix_impl {

using namespace felix_sm100::topk;

FelixCode topk_select_launch(const float* data, float* out, uint32_t num_slices,
                             uint32_t slice_size, uint32_t k, bool largest,
                             cudaStream_t stream) {
  // Argument rules of the reference launcher (sorting_radix_select_kernel_launch.cu:12-25).
  if (num_slices == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  if (!data || !out) return api_error("topk: data/out must be non-null");
  if (slice_size == 0 || k == 0 || k > slice_size)
    return api_error("topk: k must be in [1, slice_size] and slice_size > 0");
  if (num_slices > 65535u * 1024u) return api_error("topk: too many slices");
  DeviceInfo* dev = current_device_info();
  if (!dev) return launch_error(cudaGetLastError(), "topk: no CUDA device");

  // Few slices, each far larger than one CTA streams quickly: spread every
  // pass over the whole GPU.
  const bool grid_wide = num_slices < uint32_t(dev->num_sms) / 2 && slice_size >= (1u << 20) &&
                         num_slices <= 65535u;
  cudaError_t e;
  if (!grid_wide && slice_size <= kWarpKeys) {
    const uint32_t blocks = (num_slices + kWarps - 1) / kWarps;
    select_warp_per_slice_kernel<<<blocks, kThreads, 0, stream>>>(data, out, num_slices,
                                                                  slice_size, k, largest ? 1 : 0);
  } else if (!grid_wide && slice_size >= kL2MinKeys && (slice_size & 3u) == 0 &&
             (reinterpret_cast<uintptr_t>(data) & 15u) == 0) {
    // aligned slices of 8K values and more: unstaged, re-read through the L2
    // (4096 x 32768: 354 us staged, 234 us this way; 512 x 200000: 1190 us
    // with four passes from global memory, 242 us)
    const uint32_t cap = min(slice_size / 2, 8192u);
    const size_t smem = size_t(cap) * 4;
    static PerDeviceOnce once_l2;
    const int rc = once_l2.run(dev->ordinal, [] {
      return int(cudaFuncSetAttribute(select_radix3_kernel<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(kStagedDynBytes)));
    });
    if (rc < 0) return api_error("topk: device ordinal");
    if (rc > 0) return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
    select_radix3_kernel<false><<<num_slices, kThreads, smem, stream>>>(
        data, out, slice_size, k, largest ? 1 : 0, cap, dev->status_word);
  } else if (!grid_wide && slice_size <= kSmemKeys && (slice_size & 3u) == 0 &&
             (reinterpret_cast<uintptr_t>(data) & 15u) == 0) {
    // staged, bulk-copied: candidates after the slice, at most half its size
    const uint32_t room = (kStagedDynBytes - slice_size * 4u) / 4u;
    const uint32_t cap = min(slice_size / 2, room);
    const size_t smem = size_t(slice_size + cap) * 4;
    static PerDeviceOnce once_staged;
    const int rc = once_staged.run(dev->ordinal, [] {
      return int(cudaFuncSetAttribute(select_radix3_kernel<true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(kStagedDynBytes)));
    });
    if (rc < 0) return api_error("topk: device ordinal");
    if (rc > 0) return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
    select_radix3_kernel<true><<<num_slices, kThreads, smem, stream>>>(
        data, out, slice_size, k, largest ? 1 : 0, cap, dev->status_word);
  } else if (!grid_wide) {
    const int staged = slice_size <= kSmemKeys ? 1 : 0;
    const size_t smem = staged ? size_t(slice_size) * 4 : 0;
    static PerDeviceOnce once;
    const int rc = once.run(dev->ordinal, [] {
      return int(cudaFuncSetAttribute(select_per_slice_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(kSmemKeys * 4)));
    });
    if (rc < 0) return api_error("topk: device ordinal");
    if (rc > 0) return FelixCode{FELIX_API_ERROR, cudaError_t(rc)};
    select_per_slice_kernel<<<num_slices, kThreads, smem, stream>>>(
        data, out, slice_size, k, largest ? 1 : 0, staged, dev->status_word);
  } else {
    const size_t need = kWsCounterBytes + size_t(num_slices) * (256 * 4 + sizeof(SliceState));
    uint8_t* ws = static_cast<uint8_t*>(library_workspace(dev, stream, need));
    if (!ws) return launch_error(cudaErrorMemoryAllocation, "topk: workspace");
    uint32_t* hist = reinterpret_cast<uint32_t*>(ws + kWsCounterBytes);
    SliceState* state = reinterpret_cast<SliceState*>(hist + size_t(num_slices) * 256);
    e = cudaMemsetAsync(hist, 0, size_t(num_slices) * 256 * 4, stream);
    if (e != cudaSuccess) return launch_error(e, "topk: clearing histograms");
    init_state_kernel<<<(num_slices + 255) / 256, 256, 0, stream>>>(state, num_slices, slice_size,
                                                                    k, largest ? 1 : 0);
    const uint32_t per_slice = (uint32_t(dev->num_sms) * 2 + num_slices - 1) / num_slices;
    const uint32_t max_blocks = (slice_size + kThreads * 4 - 1) / (kThreads * 4);
    const dim3 grid(per_slice < max_blocks ? per_slice : max_blocks, num_slices);
    uint32_t mask = 0;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      histogram_pass_kernel<<<grid, kThreads, 0, stream>>>(data, slice_size, shift, mask, state,
                                                           hist);
      pick_pass_kernel<<<num_slices, 32, 0, stream>>>(hist, state, shift, pass == 3 ? 1 : 0, out);
      mask |= 255u << shift;
    }
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return launch_error(e, "topk: launch failed");
  return FelixCode{FELIX_SUCCESS, cudaSuccess};
}

}  // namespace felix_impl
