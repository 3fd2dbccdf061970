// Top-k token selection with a recent window (mskv_topk).
//
// Replaces torch.topk over the head-averaged scores (qwen-eljrte/Qwen_Transformer/
// attention.py:567-572) with a per-selection radix select:
//
//  * one 1024-thread CTA per selection (one (sequence, KV head) pair in per-head mode, one
//    sequence in the reference's head-averaged mode);
//  * fp32 keys are mapped to order-preserving uint32 (sign flip), and four 8-bit radix
//    passes over the candidates build a 256-bin histogram of the digit under the current
//    prefix.  Threads with equal digits are merged with __match_any_sync before one shared
//    atomic per group, because the high digits of real scores fall into a handful of bins;
//  * the pass ends knowing the exact k-th key tau and how many keys equal to tau to keep;
//  * an ordered compaction (each thread owns a contiguous run, one block-wide 64-bit scan
//    of (#greater, #equal)) writes the selected token indices in ascending order, keeping
//    ties at tau toward the lower token index, and appends the recent window.  NaN keys
//    rank highest.
// The scores are re-read from L2 on every pass (64 KB per 16k-token selection).
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
  int32_t len_scalar, k_scalar, recent, num_sel, rows_per_sel, sel_per_batch, out64;
};

// Order-preserving map fp32 -> uint32.  Every NaN (either sign, any payload) maps to the
// largest key, so NaN ranks above +inf whatever NaN encoding the arithmetic produced.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint32_t key_at(const TopkDev& a, const float* row0, int64_t t) {
  float s = row0[t];
  for (int r = 1; r < a.rows_per_sel; ++r) s += row0[(int64_t)r * a.ss + t];
  return order_key(s * a.scale);
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
  __shared__ uint32_t hist[kTkWarps][256];
  __shared__ uint32_t tot[256];
  __shared__ uint32_t s_prefix, s_krem;
  __shared__ uint64_t s_scan[kTkWarps];

  const int64_t j = blockIdx.x;
  const int b = (int)(j / a.sel_per_batch);
  const int64_t L = a.len ? (int64_t)a.len[b] : (int64_t)a.len_scalar;
  const int64_t n = L > a.recent ? L - a.recent : 0;  // candidates [0, n)
  int64_t K = a.topk ? (int64_t)a.topk[b] : (int64_t)a.k_scalar;
  if (K < 0) K = 0;
  if (K > n) K = n;
  const int64_t w = L - n;  // recent window [n, L)
  const float* row0 = a.scores + j * a.rows_per_sel * a.ss;
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
// Cluster path: 8 CTAs (one thread-block cluster) per selection.
//
// CTA r of the cluster owns the r-th eighth of the candidates and keeps their keys in shared
// memory (loaded once).  Each radix pass builds the CTA's 256-bin histogram, then every CTA
// sums the eight histograms through distributed shared memory (each pass has its own
// histogram buffer, so one cluster barrier per pass suffices) and finds the same digit.  The
// ordered compaction exchanges the per-CTA (#greater, #equal) counts the same way, so each
// CTA writes its part of the ascending output directly.
constexpr int kTcCtas = 8;
constexpr int kTcThreads = 512;
constexpr int kTcWarps = kTcThreads / 32;
constexpr int kTcMaxKeys = 16384;  // keys per CTA held in shared memory (64 KB)

template <int NW>
__device__ __forceinline__ uint64_t block_exclusive_scan_n(uint64_t v, uint64_t* warp_tot, uint64_t* total) {
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
    uint64_t w = lane < NW ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    if (lane < NW) warp_tot[lane] = w;
  }
  __syncthreads();
  *total = warp_tot[NW - 1];
  const uint64_t before_warp = warp ? warp_tot[warp - 1] : 0;
  return before_warp + inc - v;
}

__global__ void __cluster_dims__(kTcCtas, 1, 1) __launch_bounds__(kTcThreads)
    topk_cluster_kernel(const TopkDev a) {
  extern __shared__ uint32_t s_keys[];
  __shared__ uint32_t s_hist[4][256];
  __shared__ uint32_t s_tot[256];
  __shared__ uint32_t s_prefix, s_krem;
  __shared__ uint64_t s_cnt;
  __shared__ uint64_t s_scan[kTcWarps];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int64_t j = blockIdx.x / kTcCtas;
  const int b = (int)(j / a.sel_per_batch);
  const int64_t L = a.len ? (int64_t)a.len[b] : (int64_t)a.len_scalar;
  const int64_t n = L > a.recent ? L - a.recent : 0;
  int64_t K = a.topk ? (int64_t)a.topk[b] : (int64_t)a.k_scalar;
  if (K < 0) K = 0;
  if (K > n) K = n;
  const int64_t w = L - n;
  const float* row0 = a.scores + j * a.rows_per_sel * a.ss;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = (n + kTcCtas - 1) / kTcCtas;
  const int64_t lo = min((int64_t)rank * chunk, n);
  const int64_t hi = min(lo + chunk, n);
  const int m = (int)(hi - lo);

  uint32_t prefix = 0, mask = 0, krem = (uint32_t)K;
  if (K > 0 && K < n) {
    for (int i = tid; i < m; i += kTcThreads) s_keys[i] = key_at(a, row0, lo + i);
    for (int i = tid; i < 4 * 256; i += kTcThreads) (&s_hist[0][0])[i] = 0;   // one histogram per pass
    __syncthreads();
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      // histogram of this pass's digit; equal digits within a warp are merged before the atomic
      for (int base = 0; base < m; base += kTcThreads) {
        const int i = base + tid;
        uint32_t bin = 0xffffffffu;
        if (i < m) {
          const uint32_t key = s_keys[i];
          if ((key & mask) == prefix) bin = (key >> shift) & 255u;
        }
        const uint32_t peers = __match_any_sync(0xffffffffu, bin);
        if (bin != 0xffffffffu && lane == __ffs(peers) - 1) atomicAdd(&s_hist[pass][bin], __popc(peers));
      }
      cluster.sync();   // orders every CTA's histogram before the distributed reads
      if (tid < 256) {
        uint32_t s = 0;
#pragma unroll
        for (int c = 0; c < kTcCtas; ++c) s += *cluster.map_shared_rank(&s_hist[pass][tid], c);
        s_tot[tid] = s;
      }
      __syncthreads();
      if (warp == 0) {
        uint32_t c[8], lt = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) { c[i] = s_tot[lane * 8 + i]; lt += c[i]; }
        uint32_t suf = lt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += v;
        }
        uint32_t cum = suf - lt;
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
    }
    // Ordered compaction.  Thread i owns the contiguous run [i*E, (i+1)*E) of this CTA's keys.
    const int E = (m + kTcThreads - 1) / kTcThreads;
    const int i_lo = min(tid * E, m), i_hi = min(i_lo + E, m);
    uint32_t gt = 0, eq = 0;
    for (int i = i_lo; i < i_hi; ++i) {
      gt += s_keys[i] > prefix;
      eq += s_keys[i] == prefix;
    }
    uint64_t cta_total;
    const uint64_t before = block_exclusive_scan_n<kTcWarps>(((uint64_t)gt << 32) | eq, s_scan, &cta_total);
    if (tid == 0) s_cnt = cta_total;
    cluster.sync();
    uint64_t cta_before = 0;
    for (int c = 0; c < rank; ++c) cta_before += *cluster.map_shared_rank(&s_cnt, c);
    const uint64_t all_before = cta_before + before;
    const uint32_t gt_before = (uint32_t)(all_before >> 32);
    uint32_t eq_seen = (uint32_t)(all_before & 0xffffffffu);
    int64_t pos = (int64_t)gt_before + min(eq_seen, krem);
    for (int i = i_lo; i < i_hi; ++i) {
      const uint32_t key = s_keys[i];
      if (key > prefix) {
        put(a, j, pos++, lo + i);
      } else if (key == prefix) {
        if (eq_seen < krem) put(a, j, pos++, lo + i);
        ++eq_seen;
      }
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
  // len_scalar bounds every len[b]; it sizes the per-CTA key buffer of the cluster path.
  const int64_t n_max = d->len_scalar > d->recent ? (int64_t)d->len_scalar - d->recent : 0;
  const int64_t keys_per_cta = (n_max + kTcCtas - 1) / kTcCtas;
  if (keys_per_cta <= kTcMaxKeys && (int64_t)d->num_sel * kTcCtas <= 0x7fffffffLL) {
    static bool attr_set = false;  // benign race: every thread sets the same value
    if (!attr_set) {
      cudaFuncSetAttribute(topk_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kTcMaxKeys * (int)sizeof(uint32_t));
      attr_set = true;
    }
    const size_t smem = (size_t)(keys_per_cta > 0 ? keys_per_cta : 1) * sizeof(uint32_t);
    topk_cluster_kernel<<<(unsigned)(d->num_sel * kTcCtas), kTcThreads, smem, as_stream(stream)>>>(a);
    return after_launch("mskv_topk");
  }
  topk_kernel<<<d->num_sel, kTkThreads, 0, as_stream(stream)>>>(a);
  return after_launch("mskv_topk");
}
