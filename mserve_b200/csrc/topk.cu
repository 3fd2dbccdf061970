// Top-k token selection with a recent window (mskv_topk).
//
// Replaces torch.topk over the head-averaged scores (qwen-eljrte/Qwen_Transformer/
// attention.py:567-572) with an exact radix select per selection (one (sequence, KV head) pair
// in per-head mode, one sequence in the reference's head-averaged mode):
//
//  * fp32 keys (the selection's score rows summed in row order, scaled) map to order-preserving
//    uint32 (sign flip; every NaN maps to the largest key);
//  * the keys live in shared memory: one 1024-thread CTA per selection, or a cluster of 2, 4 or
//    8 CTAs each holding a share, for up to 8 x 48K candidates;
//  * digits of 12, 12 and 8 bits: the first histogram is built while the keys load, the next
//    two passes only compare and count the keys still matching; cluster CTAs sum their
//    histograms through distributed shared memory; each digit search is a block suffix scan;
//  * the pass ends knowing the exact k-th key and how many keys equal to it to keep; an ordered
//    compaction through bitmaps (a ballot pair per 32 keys, a block scan over the words) writes
//    the selected token indices in ascending order, keeping ties at the threshold toward the
//    lower token index, and appends the recent window.
// Beyond 8 x 48K candidates one CTA per selection re-reads the scores from L2 on every pass.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace mskv {

constexpr int kTkThreads = 1024;
constexpr int kTkWarps = kTkThreads / 32;

struct TopkDev {
  const float* scores;
  int64_t ss;
  char* out;
  int64_t os;
  int32_t* counts;
  const int32_t* len;
  const int32_t* topk;
  float scale;
  int32_t len_scalar, k_scalar, recent, num_sel, rows_per_sel, sel_per_batch, out64, row_block;
  int64_t sel_stride, block_stride;
};

// Order-preserving map fp32 -> uint32.  Every NaN (either sign, any payload) maps to the
// largest key, so NaN ranks above +inf whatever NaN encoding the arithmetic produced.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Summed score of token t over the selection's rows, in row order (row 0 at row0).
__device__ __forceinline__ uint32_t key_at(const TopkDev& a, const float* row0, int64_t t) {
  float s = row0[t];
  for (int r = 1; r < a.rows_per_sel; ++r)
    s += row0[(int64_t)(r / a.row_block) * a.block_stride + (int64_t)(r % a.row_block) * a.ss + t];
  return order_key(s * a.scale);
}

// Keys [0, n) of a selection into shared memory, NL independent loads in flight per thread
// (the same fp32 sum, in row order, as key_at).  With hist != NULL every key also adds one to
// hist[key >> hist_shift].
template <int NL>
__device__ __forceinline__ void load_keys(const TopkDev& a, const float* row0, int64_t lo, int n,
                                          uint32_t* s_keys, int tid, int nthreads, uint32_t* hist = nullptr,
                                          int hist_shift = 0) {
  for (int base = tid; base < n; base += NL * nthreads) {
    float v[NL];
#pragma unroll
    for (int u = 0; u < NL; ++u) {
      const int i = base + u * nthreads;
      v[u] = i < n ? row0[lo + i] : 0.f;
    }
    // rows are added in order; unrolling lets the loads of consecutive rows be in flight
    // together (the adds stay in row order)
#pragma unroll(NL >= 16 ? 2 : 4)
    for (int r = 1; r < a.rows_per_sel; ++r) {
      const float* rr = row0 + (int64_t)(r / a.row_block) * a.block_stride + (int64_t)(r % a.row_block) * a.ss;
#pragma unroll
      for (int u = 0; u < NL; ++u) {
        const int i = base + u * nthreads;
        if (i < n) v[u] += rr[lo + i];
      }
    }
#pragma unroll
    for (int u = 0; u < NL; ++u) {
      const int i = base + u * nthreads;
      if (i < n) {
        const uint32_t key = order_key(v[u] * a.scale);
        s_keys[i] = key;
        if (hist) atomicAdd(&hist[key >> hist_shift], 1u);
      }
    }
  }
}

// load_keys for a selection of one score row whose first key is 16-byte aligned: float4 loads,
// NL in flight per thread (the same keys, so the same histogram).
template <int NL>
__device__ __forceinline__ void load_keys_row4(const TopkDev& a, const float* src, int n, uint32_t* s_keys,
                                               int tid, int nthreads, uint32_t* hist, int hist_shift) {
  const int n4 = n >> 2;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  uint4* k4 = reinterpret_cast<uint4*>(s_keys);
  for (int base = tid; base < n4; base += NL * nthreads) {
    float4 v[NL];
#pragma unroll
    for (int u = 0; u < NL; ++u) {
      const int i = base + u * nthreads;
      v[u] = i < n4 ? s4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < NL; ++u) {
      const int i = base + u * nthreads;
      if (i < n4) {
        const uint4 key = make_uint4(order_key(v[u].x * a.scale), order_key(v[u].y * a.scale),
                                     order_key(v[u].z * a.scale), order_key(v[u].w * a.scale));
        k4[i] = key;
        atomicAdd(&hist[key.x >> hist_shift], 1u);
        atomicAdd(&hist[key.y >> hist_shift], 1u);
        atomicAdd(&hist[key.z >> hist_shift], 1u);
        atomicAdd(&hist[key.w >> hist_shift], 1u);
      }
    }
  }
  for (int i = 4 * n4 + tid; i < n; i += nthreads) {
    const uint32_t key = order_key(src[i] * a.scale);
    s_keys[i] = key;
    atomicAdd(&hist[key >> hist_shift], 1u);
  }
}

__device__ __forceinline__ void put(const TopkDev& a, int64_t j, int64_t pos, int64_t tok) {
  if (a.out64) reinterpret_cast<int64_t*>(a.out)[j * a.os + pos] = tok;
  else reinterpret_cast<int32_t*>(a.out)[j * a.os + pos] = (int32_t)tok;
}

// Block-wide exclusive scan of a 64-bit value (1024 threads).
__device__ __forceinline__ uint64_t block_exclusive_scan(uint64_t v, uint64_t* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint64_t w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    warp_tot[lane] = w;  // inclusive
  }
  __syncthreads();
  const uint64_t before_warp = warp ? warp_tot[warp - 1] : 0;
  return before_warp + inc - v;
}

__global__ void __launch_bounds__(kTkThreads) topk_kernel(const TopkDev a) {
  wait_for_previous_grid();  // the scores come from the kernel before (programmatic launch)
  __shared__ uint32_t hist[kTkWarps][256];
  __shared__ uint32_t tot[256];
  __shared__ uint32_t s_prefix, s_krem;
  __shared__ uint64_t s_scan[kTkWarps];

  const int64_t j = blockIdx.x;
  const int b = (int)(j / a.sel_per_batch);
  const int64_t L = a.len ? min((int64_t)a.len[b], (int64_t)a.len_scalar) : (int64_t)a.len_scalar;
  const int64_t n = L > a.recent ? L - a.recent : 0;  // candidates [0, n)
  int64_t K = a.topk ? (int64_t)a.topk[b] : (int64_t)a.k_scalar;
  if (K < 0) K = 0;
  if (K > n) K = n;
  const int64_t w = L - n;  // recent window [n, L)
  const float* row0 = a.scores + j * a.sel_stride;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  uint32_t prefix = 0, mask = 0, krem = (uint32_t)K;
  const bool radix = K > 0 && K < n;
  if (radix) {
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = threadIdx.x; i < kTkWarps * 256; i += kTkThreads) (&hist[0][0])[i] = 0;
      __syncthreads();
      for (int64_t base = 0; base < n; base += kTkThreads) {
        const int64_t t = base + threadIdx.x;
        uint32_t bin = 0xffffffffu;
        if (t < n) {
          const uint32_t key = key_at(a, row0, t);
          if ((key & mask) == prefix) bin = (key >> shift) & 255u;
        }
        const uint32_t peers = __match_any_sync(0xffffffffu, bin);
        if (bin != 0xffffffffu && lane == __ffs(peers) - 1) atomicAdd(&hist[warp][bin], __popc(peers));
      }
      __syncthreads();
      if (threadIdx.x < 256) {
        uint32_t s = 0;
#pragma unroll 8
        for (int ww = 0; ww < kTkWarps; ++ww) s += hist[ww][threadIdx.x];
        tot[threadIdx.x] = s;
      }
      __syncthreads();
      if (warp == 0) {
        uint32_t c[8], lt = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) { c[i] = tot[lane * 8 + i]; lt += c[i]; }
        uint32_t suf = lt;  // inclusive suffix sum over lanes >= lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += v;
        }
        uint32_t cum = suf - lt;  // keys in higher lanes' bins
#pragma unroll
        for (int i = 7; i >= 0; --i) {
          if (cum < krem && cum + c[i] >= krem) {
            s_prefix = prefix | ((uint32_t)(lane * 8 + i) << shift);
            s_krem = krem - cum;
          }
          cum += c[i];
        }
      }
      __syncthreads();
      prefix = s_prefix;
      krem = s_krem;
      mask |= 0xffu << shift;
      __syncthreads();
    }
  }

  // Ordered compaction of the candidates: thread i owns [i*E, min((i+1)*E, n)).
  const int64_t E = (n + kTkThreads - 1) / kTkThreads;
  const int64_t t_lo = min((int64_t)threadIdx.x * E, n);
  const int64_t t_hi = min(t_lo + E, n);
  if (K == n) {
    for (int64_t t = threadIdx.x; t < n; t += kTkThreads) put(a, j, t, t);
  } else if (K > 0) {
    uint32_t gt = 0, eq = 0;
    for (int64_t t = t_lo; t < t_hi; ++t) {
      const uint32_t key = key_at(a, row0, t);
      gt += key > prefix;
      eq += key == prefix;
    }
    const uint64_t before = block_exclusive_scan(((uint64_t)gt << 32) | eq, s_scan);
    const uint32_t gt_before = (uint32_t)(before >> 32);
    uint32_t eq_seen = (uint32_t)(before & 0xffffffffu);
    int64_t pos = (int64_t)gt_before + min(eq_seen, krem);
    for (int64_t t = t_lo; t < t_hi; ++t) {
      const uint32_t key = key_at(a, row0, t);
      if (key > prefix) {
        put(a, j, pos++, t);
      } else if (key == prefix) {
        if (eq_seen < krem) put(a, j, pos++, t);
        ++eq_seen;
      }
    }
  }
  for (int64_t i = threadIdx.x; i < w; i += kTkThreads) put(a, j, K + i, n + i);
  if (a.counts && threadIdx.x == 0) a.counts[j] = (int32_t)(K + w);
}

// ---------------------------------------------------------------------------------------
// Shared-memory path (up to kSmMaxKeys candidates per CTA): one 1024-thread CTA per selection,
// or a cluster of 2, 4 or 8 such CTAs, keeps every candidate key in shared memory.
//
// Digits of 12, 12 and 8 bits: the first pass histograms every key into 4096 bins (plain
// shared atomics; a 12-bit digit of an fp32 key spans an eighth of a binade, so real scores
// spread over many bins); the second and third passes only compare keys against the prefix
// and count the few that still match.  Each digit search is a block-wide suffix scan over the
// histogram.  The ordered compaction is the warp-ballot one of the cluster path.
constexpr int kSmThreads = 1024;
constexpr int kSmWarps = kSmThreads / 32;
constexpr int kSmMaxKeys = 48 * 1024;  // a multiple of 4: the buffer holds whole 4-key units
constexpr int kSmBins = 4096;

// Finds the bin holding the krem-th largest key (bins ordered by value) from the 4 bin counts
// c[0..3] each thread owns (bins 4t .. 4t+3); sets prefix |= bin << shift and krem to the rank
// within that bin, and full when that rank is the bin's count: every key of the bin is then
// selected, and so is every key whose digits so far are at least the prefix.  Every thread of
// the CTA calls it.
__device__ __forceinline__ void sm_digit_search(const uint32_t (&c)[4], int shift, uint32_t* s_wsuf,
                                                uint32_t* s_prefix, uint32_t* s_krem, uint32_t* s_full,
                                                uint32_t& prefix, uint32_t& krem, bool& full) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t own = c[0] + c[1] + c[2] + c[3];
  uint32_t suf = own;  // inclusive suffix over the lanes of the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += v;
  }
  if (lane == 0) s_wsuf[warp] = suf;  // warp total
  __syncthreads();
  if (warp == 0) {
    const uint32_t wt = s_wsuf[lane];
    uint32_t ws = wt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_down_sync(0xffffffffu, ws, o);
      if (lane + o < 32) ws += v;
    }
    __syncwarp();
    s_wsuf[lane] = ws - wt;  // total of the warps above
  }
  __syncthreads();
  uint32_t cum = s_wsuf[warp] + (suf - own);  // keys in bins above this thread's bins
#pragma unroll
  for (int i = 3; i >= 0; --i) {
    if (cum < krem && cum + c[i] >= krem) {   // exactly one (thread, bin) holds the krem-th key
      *s_prefix = prefix | ((uint32_t)(4 * tid + i) << shift);
      *s_krem = krem - cum;
      *s_full = cum + c[i] == krem;
    }
    cum += c[i];
  }
  __syncthreads();
  prefix = *s_prefix;
  krem = *s_krem;
  full = *s_full != 0;
}

// The thread's 4 bins of a histogram, summed over the NCTA CTAs of the cluster (distributed
// shared memory); bins at or beyond nbins count 0.
template <int NCTA>
__device__ __forceinline__ void cluster_bins(uint32_t (&c)[4], uint32_t* hist, int nbins) {
  c[0] = c[1] = c[2] = c[3] = 0;
  if (4 * (int)threadIdx.x >= nbins) return;
  const uint4 v = reinterpret_cast<const uint4*>(hist)[threadIdx.x];
  c[0] = v.x; c[1] = v.y; c[2] = v.z; c[3] = v.w;
  if constexpr (NCTA > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned me = cluster.block_rank();
#pragma unroll
    for (int r = 0; r < NCTA; ++r) {
      if ((unsigned)r == me) continue;
      const uint4 w = reinterpret_cast<const uint4*>(cluster.map_shared_rank(hist, r))[threadIdx.x];
      c[0] += w.x; c[1] += w.y; c[2] += w.z; c[3] += w.w;
    }
  }
}

template <int NCTA>
__device__ __forceinline__ void cta_group_sync() {
  if constexpr (NCTA > 1) cg::this_cluster().sync();
  else __syncthreads();
}

// One selection per NCTA CTAs (NCTA = 1, or a cluster of 2, 4 or 8 for up to NCTA x kSmMaxKeys
// candidates): CTA r holds the keys [r*chunk, (r+1)*chunk) in shared memory.  Every radix pass
// has its own histogram buffer, so no buffer is cleared while the peer CTA may still read it.
template <int NCTA>
__global__ void __launch_bounds__(kSmThreads) topk_smem_kernel(const TopkDev a) {
  wait_for_previous_grid();  // the scores come from the kernel before (programmatic launch)
  extern __shared__ __align__(16) uint32_t s_keys[];   // this CTA's keys, padded to a multiple of 4
  __shared__ __align__(16) uint32_t s_hist0[kSmBins];
  __shared__ __align__(16) uint32_t s_hist1[kSmBins];
  __shared__ __align__(16) uint32_t s_hist2[256];
  __shared__ uint32_t s_wsuf[kSmWarps];
  __shared__ uint64_t s_wcnt[kSmWarps];
  __shared__ uint64_t s_cnt;
  __shared__ uint32_t s_prefix, s_krem, s_full;

  const int rank = NCTA > 1 ? (int)cg::this_cluster().block_rank() : 0;
  const int64_t j = blockIdx.x / NCTA;
  const int b = (int)(j / a.sel_per_batch);
  // len_scalar bounds every len[b] (it sized the key buffer): a larger len[b] is clamped
  const int64_t L = a.len ? min((int64_t)a.len[b], (int64_t)a.len_scalar) : (int64_t)a.len_scalar;
  const int n = (int)(L > a.recent ? L - a.recent : 0);
  int64_t K = a.topk ? (int64_t)a.topk[b] : (int64_t)a.k_scalar;
  if (K < 0) K = 0;
  if (K > n) K = n;
  const int64_t w = L - n;
  const float* row0 = a.scores + j * a.sel_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = (n + NCTA - 1) / NCTA;
  const int lo = min(rank * chunk, n), m = min(lo + chunk, n) - lo;   // this CTA's keys [lo, lo + m)
  const uint4* keys4 = reinterpret_cast<const uint4*>(s_keys);
  const int m4 = (m + 3) >> 2;  // 4-key units; the last may be partial (its tail is masked)

  if (K > 0 && K < n) {
    for (int i = tid; i < kSmBins; i += kSmThreads) { s_hist0[i] = 0; s_hist1[i] = 0; }
    if (tid < 256) s_hist2[tid] = 0;
    __syncthreads();
    // keys into shared memory; digit 0 (bits 31..20) histogrammed on the way
    if (a.rows_per_sel == 1 && (reinterpret_cast<uintptr_t>(row0 + lo) & 15) == 0)
      load_keys_row4<4>(a, row0 + lo, m, s_keys, tid, kSmThreads, s_hist0, 20);
    else
      load_keys<16>(a, row0, lo, m, s_keys, tid, kSmThreads, s_hist0, 20);
    cta_group_sync<NCTA>();
    uint32_t prefix = 0, krem = (uint32_t)K, c[4];
    bool full = false;
    cluster_bins<NCTA>(c, s_hist0, kSmBins);
    sm_digit_search(c, 20, s_wsuf, &s_prefix, &s_krem, &s_full, prefix, krem, full);
    if (full) {
      // the bitmaps below reuse s_hist0, which the peer CTAs read for digit 0
      if constexpr (NCTA > 1) cta_group_sync<NCTA>();
    } else {
      // digit 1: bits 19..8 of the keys whose top 12 bits match
      for (int u = tid; u < m4; u += kSmThreads) {
        const uint4 kv = keys4[u];
        const uint32_t k4[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (4 * u + e < m && (k4[e] >> 20) == (prefix >> 20)) atomicAdd(&s_hist1[(k4[e] >> 8) & 0xfffu], 1u);
      }
      cta_group_sync<NCTA>();
      cluster_bins<NCTA>(c, s_hist1, kSmBins);
      sm_digit_search(c, 8, s_wsuf, &s_prefix, &s_krem, &s_full, prefix, krem, full);
    }
    if (!full) {
      // digit 2: bits 7..0 of the keys whose top 24 bits match
      for (int u = tid; u < m4; u += kSmThreads) {
        const uint4 kv = keys4[u];
        const uint32_t k4[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (4 * u + e < m && (k4[e] >> 8) == (prefix >> 8)) atomicAdd(&s_hist2[k4[e] & 0xffu], 1u);
      }
      cta_group_sync<NCTA>();
      cluster_bins<NCTA>(c, s_hist2, 256);
      sm_digit_search(c, 0, s_wsuf, &s_prefix, &s_krem, &s_full, prefix, krem, full);
    } else {
      // Stopped early: the selection is every key at or above the prefix (its unresolved low
      // bits are zero).  Some key lies below it (K < n), so prefix > 0, and "above prefix - 1,
      // no ties kept" describes the same set to the compaction.
      prefix -= 1u;
      krem = 0;
    }

    // Ordered compaction through bitmaps.  Word q covers this CTA's keys [32q, 32q+32), bit i =
    // key lo + 32q + i: G_q marks keys above the threshold key, E_q keys equal to it (one
    // ballot pair per word).  A block scan of (#G, #E) per word, offset by the counts of the
    // lower-ranked CTA, gives every word its output position and how many equal keys before it
    // were kept; its thread then writes only its selected keys.  s_hist0 holds the words: every
    // CTA finished reading the peers' digit-0 histograms before the digit-1 barrier.
    const int nw = (m + 31) >> 5;                 // <= kSmMaxKeys / 32 = 1536 words
    uint32_t* s_g = s_hist0;
    uint32_t* s_e = s_hist0 + kSmMaxKeys / 32;
    for (int q = warp; q < nw; q += kSmWarps) {
      const int i = 32 * q + lane;
      const uint32_t key = i < m ? s_keys[i] : 0u;
      const uint32_t gm = __ballot_sync(0xffffffffu, i < m && key > prefix);
      const uint32_t em = __ballot_sync(0xffffffffu, i < m && key == prefix);
      if (lane == 0) { s_g[q] = gm; s_e[q] = em; }
    }
    __syncthreads();
    // thread t owns words [t*WPT, t*WPT + WPT)
    const int WPT = (nw + kSmThreads - 1) / kSmThreads;   // 1 or 2
    const int q0 = min(tid * WPT, nw), q1 = min(q0 + WPT, nw);
    uint64_t own = 0;
    for (int q = q0; q < q1; ++q) own += ((uint64_t)__popc(s_g[q]) << 32) | (uint64_t)__popc(s_e[q]);
    uint64_t inc = own;                            // inclusive scan over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    if (lane == 31) s_wcnt[warp] = inc;
    __syncthreads();
    uint64_t before = lane < warp ? s_wcnt[lane] : 0;   // totals of the warps below
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
    before += inc - own;
    if constexpr (NCTA > 1) {
      if (tid == 0) {
        uint64_t tot = 0;
        for (int v = 0; v < kSmWarps; ++v) tot += s_wcnt[v];
        s_cnt = tot;
      }
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      for (int r = 0; r < rank; ++r) before += *cluster.map_shared_rank(&s_cnt, r);
    }
    uint32_t gtb = (uint32_t)(before >> 32), eqb = (uint32_t)(before & 0xffffffffu);
    for (int q = q0; q < q1; ++q) {
      const uint32_t gm = s_g[q], em = s_e[q];
      // keep the first (krem - eqb) equal keys, in token order
      uint32_t keep = 0, rest = em;
      for (uint32_t r = eqb; r < krem && rest; ++r) {
        const uint32_t low = rest & (0u - rest);
        keep |= low;
        rest ^= low;
      }
      uint32_t sel = gm | keep;
      int64_t pos = (int64_t)gtb + min(eqb, krem);
      while (sel) {
        const int bit = __ffs(sel) - 1;
        put(a, j, pos++, lo + 32 * q + bit);
        sel &= sel - 1;
      }
      gtb += __popc(gm);
      eqb += __popc(em);
    }
  } else if (K == n) {
    for (int t = lo + tid; t < lo + m; t += kSmThreads) put(a, j, t, t);
  }
  if (rank == 0) {
    for (int64_t i = tid; i < w; i += kSmThreads) put(a, j, K + i, n + i);
    if (a.counts && tid == 0) a.counts[j] = (int32_t)(K + w);
  }
  if constexpr (NCTA > 1) cg::this_cluster().sync();  // no CTA leaves while its peer may read its memory
}

// ---------------------------------------------------------------------------------------
// Cluster path: 8 CTAs (one thread-block cluster) per selection.
//
// CTA r of the cluster owns the r-th eighth of the candidates and keeps their keys in shared
// memory.  The first digit's histogram is built while the keys are loaded.  Each radix pass
// ends with every CTA summing the eight histograms through distributed shared memory (one
// buffer per pass, so one cluster barrier per pass) and finding the same digit with a
// 256-thread suffix scan.  Passes 1-3 visit only the keys that still match the prefix: pass 1
// appends the keys matching the first digit to a survivor list, pass 2 filters that list
// again, so the last passes touch a handful of keys.  The ordered compaction gives each warp a
// contiguous run of keys, counts with ballots, exchanges the per-CTA (#greater, #equal)
// counts through distributed shared memory and writes the ascending output directly.
constexpr int kTcCtas = 8;
constexpr int kTcThreads = 512;
constexpr int kTcWarps = kTcThreads / 32;
constexpr int kTcMaxKeys = 16384;  // keys per CTA; shared memory holds them plus two survivor lists

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Histogram of one digit (bin 0xffffffff = no contribution).  Plain shared atomics: merging
// equal digits of a warp with __match_any_sync first was slower on both spread-out and
// tie-heavy scores.
__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin, int) {
  if (bin != 0xffffffffu) atomicAdd(&hist[bin], 1u);
}

// Appends `key` to list[*count] for lanes with keep set (warp-aggregated).
__device__ __forceinline__ void list_push(uint32_t* list, uint32_t* count, bool keep, uint32_t key, int lane) {
  const uint32_t bal = __ballot_sync(0xffffffffu, keep);
  if (!bal) return;
  uint32_t base = 0;
  if (lane == 0) base = atomicAdd(count, (uint32_t)__popc(bal));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (keep) list[base + __popc(bal & lanemask_lt())] = key;
}

__global__ void __cluster_dims__(kTcCtas, 1, 1) __launch_bounds__(kTcThreads)
    topk_cluster_kernel(const TopkDev a, int cap) {
  wait_for_previous_grid();  // the scores come from the kernel before (programmatic launch)
  extern __shared__ uint32_t s_dyn[];
  __shared__ uint32_t s_hist[4][256];
  __shared__ uint32_t s_wsuf[8];
  __shared__ uint32_t s_prefix, s_krem, s_n1, s_n2;
  __shared__ uint64_t s_wcnt[kTcWarps];
  __shared__ uint64_t s_cnt;
  uint32_t* s_keys = s_dyn;            // this CTA's keys, in token order
  uint32_t* s_l1 = s_dyn + cap;        // keys matching the first digit
  uint32_t* s_l2 = s_dyn + 2 * cap;    // keys matching the first two digits

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int64_t j = blockIdx.x / kTcCtas;
  const int b = (int)(j / a.sel_per_batch);
  // len_scalar bounds every len[b] (it sized the key buffers): a larger len[b] is clamped
  const int64_t L = a.len ? min((int64_t)a.len[b], (int64_t)a.len_scalar) : (int64_t)a.len_scalar;
  const int64_t n = L > a.recent ? L - a.recent : 0;
  int64_t K = a.topk ? (int64_t)a.topk[b] : (int64_t)a.k_scalar;
  if (K < 0) K = 0;
  if (K > n) K = n;
  const int64_t w = L - n;
  const float* row0 = a.scores + j * a.sel_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = (n + kTcCtas - 1) / kTcCtas;
  const int64_t lo = min((int64_t)rank * chunk, n);
  const int64_t hi = min(lo + chunk, n);
  const int m = (int)(hi - lo);

  if (K > 0 && K < n) {
    for (int i = tid; i < 4 * 256; i += kTcThreads) (&s_hist[0][0])[i] = 0;
    if (tid == 0) { s_n1 = 0; s_n2 = 0; }
    __syncthreads();
    load_keys<8>(a, row0, lo, m, s_keys, tid, kTcThreads);
    // first digit's histogram: each thread reads back the keys it stored itself
    for (int base = 0; base < m; base += kTcThreads) {
      const int i = base + tid;
      hist_add(s_hist[0], i < m ? s_keys[i] >> 24 : 0xffffffffu, lane);
    }
    uint32_t prefix = 0, krem = (uint32_t)K;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      if (pass > 0) {
        const uint32_t mask = 0xffffffffu << (shift + 8);
        if (pass == 1) {          // all keys; survivors of digit 0 go to list 1
          for (int base = 0; base < m; base += kTcThreads) {
            const int i = base + tid;
            const uint32_t key = i < m ? s_keys[i] : 0u;
            const bool keep = i < m && (key & mask) == prefix;
            hist_add(s_hist[1], keep ? (key >> shift) & 255u : 0xffffffffu, lane);
            list_push(s_l1, &s_n1, keep, key, lane);
          }
        } else if (pass == 2) {   // list 1; survivors of digits 0-1 go to list 2
          const int n1 = (int)s_n1;
          for (int base = 0; base < n1; base += kTcThreads) {
            const int i = base + tid;
            const uint32_t key = i < n1 ? s_l1[i] : 0u;
            const bool keep = i < n1 && (key & mask) == prefix;
            hist_add(s_hist[2], keep ? (key >> shift) & 255u : 0xffffffffu, lane);
            list_push(s_l2, &s_n2, keep, key, lane);
          }
        } else {                  // list 2
          const int n2 = (int)s_n2;
          for (int base = 0; base < n2; base += kTcThreads) {
            const int i = base + tid;
            const uint32_t key = i < n2 ? s_l2[i] : 0u;
            const bool keep = i < n2 && (key & mask) == prefix;
            hist_add(s_hist[3], keep ? key & 255u : 0xffffffffu, lane);
          }
        }
      }
      cluster.sync();   // every CTA's histogram (and this CTA's lists) complete
      // digit search: bin t's count summed over the cluster; suffix sums over higher bins
      uint32_t c = 0, suf = 0;
      if (tid < 256) {
#pragma unroll
        for (int r = 0; r < kTcCtas; ++r) c += *cluster.map_shared_rank(&s_hist[pass][tid], r);
        suf = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += v;
        }
        if (lane == 0) s_wsuf[warp] = suf;
      }
      __syncthreads();
      if (tid < 256) {
        uint32_t above = suf - c;
        for (int w2 = warp + 1; w2 < 8; ++w2) above += s_wsuf[w2];
        if (above < krem && above + c >= krem) {
          s_prefix = prefix | ((uint32_t)tid << shift);
          s_krem = krem - above;
        }
      }
      __syncthreads();
      prefix = s_prefix;
      krem = s_krem;
    }
    // Ordered compaction.  Warp v owns the contiguous run [v*R, (v+1)*R) of this CTA's keys.
    const int R = ((m + kTcThreads - 1) / kTcThreads) * 32;
    const int w_lo = min(warp * R, m), w_hi = min(w_lo + R, m);
    uint32_t gt = 0, eq = 0;
    for (int base = w_lo; base < w_hi; base += 32) {
      const int i = base + lane;
      const uint32_t key = i < w_hi ? s_keys[i] : 0u;
      gt += __popc(__ballot_sync(0xffffffffu, i < w_hi && key > prefix));
      eq += __popc(__ballot_sync(0xffffffffu, i < w_hi && key == prefix));
    }
    if (lane == 0) s_wcnt[warp] = ((uint64_t)gt << 32) | eq;
    __syncthreads();
    uint64_t warp_before = 0, cta_total = 0;
    for (int v = 0; v < kTcWarps; ++v) {
      const uint64_t x = s_wcnt[v];
      if (v < warp) warp_before += x;
      cta_total += x;
    }
    if (tid == 0) s_cnt = cta_total;
    cluster.sync();
    uint64_t before = warp_before;
    for (int r = 0; r < rank; ++r) before += *cluster.map_shared_rank(&s_cnt, r);
    uint32_t gtb = (uint32_t)(before >> 32), eqb = (uint32_t)(before & 0xffffffffu);
    const uint32_t lt = lanemask_lt();
    for (int base = w_lo; base < w_hi; base += 32) {
      const int i = base + lane;
      const uint32_t key = i < w_hi ? s_keys[i] : 0u;
      const bool g = i < w_hi && key > prefix;
      const bool e = i < w_hi && key == prefix;
      const uint32_t bg = __ballot_sync(0xffffffffu, g), be = __ballot_sync(0xffffffffu, e);
      const uint32_t my_gt = gtb + __popc(bg & lt), my_eq = eqb + __popc(be & lt);
      if (g || (e && my_eq < krem)) put(a, j, (int64_t)my_gt + min(my_eq, krem), lo + i);
      gtb += __popc(bg);
      eqb += __popc(be);
    }
  } else if (K == n) {
    for (int64_t t = lo + tid; t < hi; t += kTcThreads) put(a, j, t, t);
  }
  if (rank == 0) {
    for (int64_t i = tid; i < w; i += kTcThreads) put(a, j, K + i, n + i);
    if (a.counts && tid == 0) a.counts[j] = (int32_t)(K + w);
  }
  cluster.sync();  // no CTA leaves while others may still read its shared memory
}

}  // namespace mskv

using namespace mskv;

extern "C" int mskv_topk(const mskv_topk_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_topk: NULL descriptor");
  if (d->num_sel < 0 || d->rows_per_sel <= 0 || d->sel_per_batch <= 0 || d->recent < 0 ||
      d->top_k_scalar < 0 || d->len_scalar < 0)
    return fail(MSKV_ERR_ARG, "mskv_topk: bad sizes");
  if (d->out_bits != 32 && d->out_bits != 64) return fail(MSKV_ERR_ARG, "mskv_topk: out_bits must be 32 or 64");
  if (d->num_sel == 0) return MSKV_OK;
  if (!d->scores || !d->out_idx) return fail(MSKV_ERR_ARG, "mskv_topk: NULL scores/out_idx");
  TopkDev a{};
  a.scores = d->scores; a.ss = d->scores_stride;
  a.out = static_cast<char*>(d->out_idx); a.os = d->out_stride;
  a.counts = d->counts; a.len = d->len; a.topk = d->top_k; a.scale = d->scale;
  a.len_scalar = d->len_scalar; a.k_scalar = d->top_k_scalar; a.recent = d->recent;
  a.num_sel = d->num_sel; a.rows_per_sel = d->rows_per_sel; a.sel_per_batch = d->sel_per_batch;
  a.out64 = d->out_bits == 64;
  if (d->row_block < 0 || d->sel_stride < 0 || d->block_stride < 0)
    return fail(MSKV_ERR_ARG, "mskv_topk: negative row layout");
  a.row_block = d->row_block > 0 ? d->row_block : d->rows_per_sel;
  a.sel_stride = d->sel_stride > 0 ? d->sel_stride : (int64_t)d->rows_per_sel * d->scores_stride;
  a.block_stride = d->block_stride;
  // len_scalar bounds every len[b]; it sizes the per-CTA key buffers.
  const int64_t n_max = d->len_scalar > d->recent ? (int64_t)d->len_scalar - d->recent : 0;
  // Which kernel (all measured on the decode shapes):
  //  * up to 2 x kSmMaxKeys candidates: the shared-memory kernel, one CTA per selection, or a
  //    2-CTA cluster beyond kSmMaxKeys;
  //  * few selections that each sum several rows over many tokens (a head-averaged selection),
  //    or up to 8 x kTcMaxKeys candidates: the 8-CTA cluster kernel (one CTA per selection would
  //    stream rows x tokens x 4 bytes through a single SM; the shared-memory kernel split eight
  //    ways spends more on its 4096-bin histograms than it saves);
  //  * longer contexts, up to 8 x kSmMaxKeys: the shared-memory kernel as a 4- or 8-CTA cluster;
  //  * beyond that: one CTA per selection re-reading the scores from L2.
  const bool wide_load = d->rows_per_sel >= 4 && n_max >= 8192 && (int64_t)d->num_sel * kTcCtas <= 2 * num_sms();
  const int64_t keys_per_cta = (n_max + kTcCtas - 1) / kTcCtas;
  const bool cluster_path = keys_per_cta <= kTcMaxKeys && (wide_load || n_max > 2 * (int64_t)kSmMaxKeys);
  int ncta = 0;
  if (!cluster_path)
    for (int c : {1, 2, 4, 8})
      if (!ncta && (n_max + c - 1) / c <= kSmMaxKeys) ncta = c;
  if (cluster_path && (int64_t)d->num_sel * kTcCtas <= 0x7fffffffLL) {
    int rc = ensure_smem_limit((const void*)topk_cluster_kernel, 3 * kTcMaxKeys * (int)sizeof(uint32_t), "mskv_topk");
    if (rc) return rc;
    const int cap = (int)(keys_per_cta > 0 ? keys_per_cta : 1);
    const size_t smem = 3 * (size_t)cap * sizeof(uint32_t);
    const cudaError_t e = launch_dependent(topk_cluster_kernel, dim3((unsigned)(d->num_sel * kTcCtas)),
                                           dim3(kTcThreads), smem, as_stream(stream), a, cap);
    if (e != cudaSuccess) return cuda_status(e, "mskv_topk launch");
    return after_launch("mskv_topk");
  }
  if (ncta && (int64_t)d->num_sel * ncta <= 0x7fffffffLL) {
    const int64_t per_cta = (n_max + ncta - 1) / ncta;
    const size_t smem = (size_t)((per_cta + 3) / 4 * 4 + (per_cta == 0 ? 4 : 0)) * sizeof(uint32_t);
    const void* kern = ncta == 1 ? (const void*)topk_smem_kernel<1>
                     : ncta == 2 ? (const void*)topk_smem_kernel<2>
                     : ncta == 4 ? (const void*)topk_smem_kernel<4> : (const void*)topk_smem_kernel<8>;
    int rc = ensure_smem_limit(kern, kSmMaxKeys * (int)sizeof(uint32_t), "mskv_topk");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(d->num_sel * ncta));
    cfg.blockDim = dim3(kSmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = ncta;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ncta == 1 ? 1 : 2;      // the one-CTA kernel is launched without a cluster
    cudaError_t e;
    switch (ncta) {
      case 1: e = cudaLaunchKernelEx(&cfg, topk_smem_kernel<1>, a); break;
      case 2: e = cudaLaunchKernelEx(&cfg, topk_smem_kernel<2>, a); break;
      case 4: e = cudaLaunchKernelEx(&cfg, topk_smem_kernel<4>, a); break;
      default: e = cudaLaunchKernelEx(&cfg, topk_smem_kernel<8>, a); break;
    }
    if (e != cudaSuccess) return cuda_status(e, "mskv_topk launch");
    return after_launch("mskv_topk");
  }
  // beyond 8 x kSmMaxKeys candidates: one CTA per selection re-reading the scores from L2
  const cudaError_t e = launch_dependent(topk_kernel, dim3((unsigned)d->num_sel), dim3(kTkThreads), 0,
                                         as_stream(stream), a);
  if (e != cudaSuccess) return cuda_status(e, "mskv_topk launch");
  return after_launch("mskv_topk");
}
