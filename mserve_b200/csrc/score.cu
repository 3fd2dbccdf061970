// Importance scoring of every cached token against the decode query (mskv_score).
//
// The reference computes torch.matmul(q, Kᵀ) over repeat_kv'd heads and averages over all
// query heads (qwen-eljrte/Qwen_Transformer/attention.py:558-565).  Here the GQA group is
// folded first: sum_g q_g·k = (sum_g q_g)·k, so every K element is read once from HBM and
// costs one FMA.  The kernels are memory-bound GEMVs (tensor cores are deliberately unused).
// 16-bit keys with head_dim 64/128/256 take score_stream_kernel (below); fp32 keys take
// score_fast_kernel; any other shape the generic one-warp-per-row kernel.
//
// score_fast_kernel:
//  * a group of GL lanes (GL = 16 for bf16 D=128) owns GL consecutive rows per iteration;
//    lane l loads the l-th 16-byte chunk of each of those rows (GL independent 16-byte loads
//    in flight per lane, 256 contiguous bytes per row per instruction), converts to fp32 and
//    accumulates one partial dot product per row;
//  * a butterfly reduce-scatter over the GL lanes (GL-1 shuffles for GL rows instead of
//    GL*log2(GL)) leaves lane l holding the full fp32 score of row l, so a warp writes its
//    32 scores as one coalesced 128-byte store;
//  * warps own contiguous runs of 32-row slices, so the GQA-summed query is rebuilt only when
//    a warp crosses into a new (b, KV head) segment.
#include <type_traits>

#include "common.cuh"

namespace mskv {

struct ScoreDev {
  RowsDev k;
  const char* q;
  int64_t q_sb, q_sh;
  float* scores;
  int64_t scores_stride;
  int64_t max_tokens;
  int32_t batch, q_heads, kv_heads, head_dim, method;
  int64_t slices_per_seg;
  int64_t total_slices;
  int64_t slices_per_warp;
  int32_t page_shift;       // log2(page_size) when it is a power of two, else -1
  int32_t npeers;           // other ranks' copies of the score rows (mskv_score_fanout), 0..7
  float* peers[kMaxPeers];  // each at the same offsets as `scores`, in another GPU's memory
};

// One score: this rank's row and, with fan-out, the same element of every peer's copy (a
// plain store through the peer mapping, over NVLink).
__device__ __forceinline__ void put_score(const ScoreDev& a, int64_t i, float v) {
  a.scores[i] = v;
  for (int p = 0; p < a.npeers; ++p) a.peers[p][i] = v;
}

// With fan-out, a writing thread's stores are made visible to the whole system before it
// exits, so a flag written after this kernel (mskv_flag_signal) orders them for the peers.
__device__ __forceinline__ void publish_scores(const ScoreDev& a) {
  if (a.npeers) __threadfence_system();
}

template <typename T> struct Cvt;
template <> struct Cvt<__nv_bfloat16> {
  static constexpr int EPV = 8;
  __device__ __forceinline__ static void to_f32(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Cvt<__half> {
  static constexpr int EPV = 8;
  __device__ __forceinline__ static void to_f32(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h;
      memcpy(&h, &w[i], 4);
      const float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
};
template <> struct Cvt<float> {
  static constexpr int EPV = 4;
  __device__ __forceinline__ static void to_f32(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
};

template <typename T> __device__ __forceinline__ float load_f32(const char* p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(p);
  else if constexpr (std::is_same<T, __half>::value) return __half2float(*reinterpret_cast<const __half*>(p));
  else return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
}

// Butterfly reduce-scatter: N lanes each hold N partial values; afterwards lane (l mod N)
// holds the sum over the N lanes of value l.
template <int N>
__device__ __forceinline__ float reduce_scatter(float (&v)[N], int lane) {
#pragma unroll
  for (int o = N / 2; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < o; ++j) {
      const float send = upper ? v[j] : v[j + o];
      const float keep = upper ? v[j + o] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// Fast path: 16-byte vectors, D/EPV lanes per row, rows of a group iteration contiguous in
// memory (strided K, or paged K with page_size a multiple of GL).
template <typename T, int D, int METHOD, bool PAGED>
__global__ void __launch_bounds__(256) score_fast_kernel(const ScoreDev a) {
  allow_dependents();  // the top-k kernel may become resident as this grid drains
  constexpr int EPV = Cvt<T>::EPV;
  constexpr int LPR = D / EPV;              // 16-byte chunks per row
  constexpr int GL = LPR < 16 ? LPR : 16;   // lanes per group (rows per group iteration)
  constexpr int VPL = LPR / GL;             // chunks per lane per row
  static_assert(LPR % GL == 0 && GL >= 2 && GL <= 16, "unsupported head_dim");

  const int lane = threadIdx.x & 31;
  const int gl = lane & (GL - 1);           // lane within group
  const int grp = lane / GL;                // group within warp
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t s_begin = warp * a.slices_per_warp;
  const int64_t s_end = min(s_begin + a.slices_per_warp, a.total_slices);

  float qs[VPL][EPV];
  int64_t cur_seg = -1;
  int b = 0, h = 0;
  int64_t len = 0;
  for (int64_t s = s_begin; s < s_end; ++s) {
    const int64_t seg = s / a.slices_per_seg;
    const int64_t t_slice = (s - seg * a.slices_per_seg) * 32;
    if (seg != cur_seg) {
      cur_seg = seg;
      b = (int)(seg / a.kv_heads);
      h = (int)(seg - (int64_t)b * a.kv_heads);
      len = rows_len(a.k, b);
      if constexpr (METHOD == 0) {
        const int G = a.q_heads / a.kv_heads;
#pragma unroll
        for (int v = 0; v < VPL; ++v)
#pragma unroll
          for (int e = 0; e < EPV; ++e) qs[v][e] = 0.f;
        for (int g = 0; g < G; ++g) {
          const char* qrow = a.q + (int64_t)b * a.q_sb + (int64_t)(h * G + g) * a.q_sh;
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            const uint4 raw = *reinterpret_cast<const uint4*>(qrow + (int64_t)(gl + v * GL) * 16);
            float f[EPV];
            Cvt<T>::to_f32(raw, f);
#pragma unroll
            for (int e = 0; e < EPV; ++e) qs[v][e] += f[e];
          }
        }
      }
    }
    if (t_slice >= len) continue;
    const int64_t t0 = t_slice + grp * GL;  // first row of this group
    // Byte offset of row t0 (rows t0..t0+GL-1 are contiguous with stride st).
    int64_t off0 = 0;
    bool group_ok = t0 < len;
    if (group_ok) {
      if constexpr (PAGED) {
        const int64_t pidx = t0 / a.k.page_size;
        const int32_t page = a.k.page_table[(int64_t)b * a.k.pt_stride + pidx];
        group_ok = page >= 0 && page < a.k.num_pages;
        off0 = (int64_t)page * a.k.sp + (int64_t)h * a.k.sh + (t0 - pidx * a.k.page_size) * a.k.st;
      } else {
        off0 = (int64_t)b * a.k.sb + (int64_t)h * a.k.sh + t0 * a.k.st;
      }
    }
    uint4 raw[GL][VPL];
#pragma unroll
    for (int j = 0; j < GL; ++j)
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        raw[j][v] = make_uint4(0, 0, 0, 0);
        if (group_ok && t0 + j < len)
          raw[j][v] = *reinterpret_cast<const uint4*>(a.k.base_k + off0 + (int64_t)j * a.k.st +
                                                       (int64_t)(gl + v * GL) * 16);
      }
    float part[GL];
#pragma unroll
    for (int j = 0; j < GL; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        float f[EPV];
        Cvt<T>::to_f32(raw[j][v], f);
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
          if constexpr (METHOD == 0) acc = fmaf(qs[v][e], f[e], acc);
          else acc = fmaf(f[e], f[e], acc);
        }
      }
      part[j] = acc;
    }
    float score = reduce_scatter<GL>(part, gl);
    if constexpr (METHOD == 1) score = sqrtf(score);
    const int64_t t = t_slice + lane;
    if (group_ok && t < len) put_score(a, seg * a.scores_stride + t, score);
  }
  publish_scores(a);
}

// Main path for 16-bit keys: register streaming, 8 rows per lane group.
//
// GL = D/8 lanes own one row (one 16-byte chunk each); a group of GL lanes takes 8
// consecutive rows per slice, so every lane issues 8 independent 16-byte loads per slice
// (ld.global.nc with L1 bypass and a 256-byte L2 prefetch: one bf16 row) into one register
// buffer: 80 registers, 3 CTAs (24 warps) per SM, the other warps' loads in flight while a
// warp scores.  (Measured at the 7B and 32B decode shapes: 24 single-buffered warps per SM
// beat 16 double-buffered ones by 2.5-4%; fewer warps with deeper buffers, shared-memory
// staging by bulk copies or cp.async, and L2 prefetching were all slower.)  Products use
// packed fp32x2 FMAs (two lanes of fp32 per instruction); the 8 partial dots are
// reduce-scattered over 8 lanes and finished with xor-shuffles.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void ffma2(float2& acc, const float2 a, const float2 b) {
  acc = __ffma2_rn(a, b, acc);  // one packed fp32x2 FMA (sm_100)
}

template <typename T>
__device__ __forceinline__ float2 pair_f32(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  } else {
    __half2 h;
    memcpy(&h, &w, 4);
    return __half22float2(h);
  }
}

template <int NV, int M>
__device__ __forceinline__ void reduce_scatter_n(float (&v)[NV], int lane_in_group) {
  int c = NV;
#pragma unroll
  for (int o = M / 2; o >= 1; o >>= 1) {
    const bool upper = (lane_in_group & o) != 0;
    const int h = c / 2;
#pragma unroll
    for (int j = 0; j < NV / 2; ++j) {
      if (j < h) {
        const float send = upper ? v[j] : v[j + h];
        const float keep = upper ? v[j + h] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    c = h;
  }
}

// One 8-row group of a 16/32/8-row slice: where its rows are and whether they exist.
struct SliceRef {
  int64_t seg, t0, len, off0;
  int b, h;
  bool live;  // the slice starts before the segment's end (warp-uniform)
  bool ok;    // this lane group has rows and their page is mapped
};

// A warp's position in its run of slices: segment (b, h), slice index within it, and the
// sequence's length and live slice count.  Only slices that hold tokens ("live": sequence b
// has ceil(min(len_b, max_tokens) / RPW) per KV head) are numbered, so every warp gets an equal
// share of real work however ragged the lengths are; the fields are updated incrementally.
struct SliceCursor {
  int64_t seg;
  int len, live, sis;   // tokens per sequence fit in 31 bits (max_tokens is checked on the host)
  int b, h;
};

template <int RPW>
__device__ __forceinline__ int live_slices(const ScoreDev& a, int b, int* len_out = nullptr) {
  int64_t len = rows_len(a.k, b);
  len = len < 0 ? 0 : (len > a.max_tokens ? a.max_tokens : len);   // max_tokens bounds the scores rows
  if (len_out) *len_out = (int)len;
  return (int)((len + RPW - 1) / RPW);
}

// Warp-collective: this warp's share [begin, begin + count) of the live slices of the grid,
// and the cursor at its first slice.  Returns false for a warp without work.
template <int RPW>
__device__ __forceinline__ bool cursor_init(const ScoreDev& a, int64_t warp, int64_t nwarps, SliceCursor& c,
                                            int64_t& count) {
  const int lane = threadIdx.x & 31;
  if (a.batch <= 32) {                         // one pass: lane b holds sequence b
    int len_b = 0;
    const int live_b = lane < a.batch ? live_slices<RPW>(a, lane, &len_b) : 0;
    const int64_t v = (int64_t)live_b * a.kv_heads;
    int64_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    const int64_t total = __shfl_sync(0xffffffffu, inc, 31);
    const int64_t per = (total + nwarps - 1) / nwarps;
    const int64_t begin = warp * per;
    const int64_t end = min(begin + per, total);
    if (begin >= end) return false;
    count = end - begin;
    const int l = __ffs(__ballot_sync(0xffffffffu, inc > begin)) - 1;
    const int64_t off = begin - __shfl_sync(0xffffffffu, inc - v, l);
    c.b = l;
    c.live = __shfl_sync(0xffffffffu, live_b, l);
    c.len = __shfl_sync(0xffffffffu, len_b, l);
    c.h = (int)(off / c.live);
    c.sis = (int)(off - (int64_t)c.h * c.live);
    c.seg = (int64_t)c.b * a.kv_heads + c.h;
    return true;
  }
  int64_t total = 0;
  for (int b0 = 0; b0 < a.batch; b0 += 32) {
    const int b = b0 + lane;
    int64_t v = b < a.batch ? (int64_t)live_slices<RPW>(a, b) * a.kv_heads : 0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    total += v;
  }
  const int64_t per = (total + nwarps - 1) / nwarps;
  const int64_t begin = warp * per;
  const int64_t end = min(begin + per, total);
  if (begin >= end) return false;
  count = end - begin;
  int64_t base = 0;
  for (int b0 = 0; b0 < a.batch; b0 += 32) {
    const int b = b0 + lane;
    const int64_t v = b < a.batch ? (int64_t)live_slices<RPW>(a, b) * a.kv_heads : 0;
    int64_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    const int64_t chunk_total = __shfl_sync(0xffffffffu, inc, 31);
    if (begin < base + chunk_total) {            // warp-uniform
      const int l = __ffs(__ballot_sync(0xffffffffu, base + inc > begin)) - 1;
      const int64_t before = base + __shfl_sync(0xffffffffu, inc - v, l);
      c.b = b0 + l;
      c.live = live_slices<RPW>(a, c.b, &c.len);
      const int64_t off = begin - before;
      c.h = (int)(off / c.live);
      c.sis = (int)(off - (int64_t)c.h * c.live);
      c.seg = (int64_t)c.b * a.kv_heads + c.h;
      return true;
    }
    base += chunk_total;
  }
  return false;
}

template <int RPW>
__device__ __forceinline__ void cursor_next(const ScoreDev& a, SliceCursor& c) {
  if (++c.sis < c.live) return;
  c.sis = 0;
  if (++c.h < a.kv_heads) {
    ++c.seg;
    return;
  }
  c.h = 0;
  do {                                           // the next sequence that holds tokens
    ++c.b;
    c.live = c.b < a.batch ? live_slices<RPW>(a, c.b, &c.len) : 1;
  } while (c.live == 0);
  c.seg = (int64_t)c.b * a.kv_heads;
}

template <int D, bool PAGED>
__device__ __forceinline__ SliceRef locate_slice(const ScoreDev& a, const SliceCursor& c, int grp) {
  constexpr int RPW = 8 * (32 / (D / 8));
  SliceRef r;
  r.seg = c.seg;
  r.b = c.b;
  r.h = c.h;
  r.len = c.len;
  const int64_t t_slice = (int64_t)c.sis * RPW;
  r.live = t_slice < r.len;
  r.t0 = t_slice + grp * 8;
  r.ok = r.t0 < r.len;
  r.off0 = 0;
  if (r.ok) {
    if constexpr (PAGED) {
      const int64_t pidx = a.page_shift >= 0 ? (r.t0 >> a.page_shift) : r.t0 / a.k.page_size;
      const int32_t page = a.k.page_table[(int64_t)r.b * a.k.pt_stride + pidx];
      r.ok = page >= 0 && page < a.k.num_pages;
      r.off0 = (int64_t)page * a.k.sp + (int64_t)r.h * a.k.sh + (r.t0 - pidx * a.k.page_size) * a.k.st;
    } else {
      r.off0 = (int64_t)r.b * a.k.sb + (int64_t)r.h * a.k.sh + r.t0 * a.k.st;
    }
  }
  return r;
}

__device__ __forceinline__ void issue_rows(const ScoreDev& a, const SliceRef& r, int gl, uint4 (&raw)[8]) {
  const char* p = a.k.base_k + r.off0 + gl * 16;
  if (r.ok && r.t0 + 8 <= r.len) {          // a whole group: no per-row checks
#pragma unroll
    for (int j = 0; j < 8; ++j) raw[j] = ldg_stream(p + (int64_t)j * a.k.st);
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    raw[j] = make_uint4(0, 0, 0, 0);
    if (r.ok && r.t0 + j < r.len) raw[j] = ldg_stream(p + (int64_t)j * a.k.st);
  }
}

template <typename T, int D, int METHOD>
__device__ __forceinline__ void score_rows(const ScoreDev& a, const SliceRef& r, int gl, const float2 (&qs)[4],
                                           const uint4 (&raw)[8]) {
  constexpr int GL = D / 8;
  float part[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = pair_f32<T>(w[i]);
      if constexpr (METHOD == 0) ffma2(acc, qs[i], f);
      else ffma2(acc, f, f);
    }
    part[j] = acc.x + acc.y;
  }
  reduce_scatter_n<8, 8>(part, gl & 7);
  float sc = part[0];
#pragma unroll
  for (int o = 8; o < GL; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
  if constexpr (METHOD == 1) sc = sqrtf(sc);
  const int64_t t = r.t0 + (gl & 7);
  if (gl < 8 && t < r.len) put_score(a, r.seg * a.scores_stride + t, r.ok ? sc : -INFINITY);
}

template <typename T>
__device__ __forceinline__ void gqa_query(const ScoreDev& a, int b, int h, int gl, float2 (&qs)[4]) {
  const int G = a.q_heads / a.kv_heads;
#pragma unroll
  for (int i = 0; i < 4; ++i) qs[i] = make_float2(0.f, 0.f);
  for (int g = 0; g < G; ++g) {
    const uint4 raw =
        *reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.q_sb + (int64_t)(h * G + g) * a.q_sh + gl * 16);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = pair_f32<T>(w[i]);
      qs[i].x += f.x;
      qs[i].y += f.y;
    }
  }
}

// Each warp walks its contiguous run of slices: the 8 loads of a slice, then its score.
template <typename T, int D, int METHOD, bool PAGED>
__global__ void __launch_bounds__(256, 3) score_stream_kernel(const ScoreDev a) {
  allow_dependents();  // the top-k kernel may become resident as this grid drains
  constexpr int GL = D / 8;
  static_assert(GL >= 8 && GL <= 32, "head_dim must be 64, 128 or 256");
  const int lane = threadIdx.x & 31;
  const int gl = lane % GL, grp = lane / GL;
  constexpr int RPW = 8 * (32 / GL);
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  SliceCursor cur_pos;
  int64_t count = 0;
  if (!cursor_init<RPW>(a, warp, nwarps, cur_pos, count)) return;
  float2 qs[4];
  int64_t q_seg = -1;
  auto score = [&](const SliceRef& r, const uint4 (&raw)[8]) {
    if (!r.live) return;  // warp-uniform
    if constexpr (METHOD == 0) {
      if (r.seg != q_seg) {
        q_seg = r.seg;
        gqa_query<T>(a, r.b, r.h, gl, qs);
      }
    }
    score_rows<T, D, METHOD>(a, r, gl, qs, raw);
  };

  uint4 buf[8];
  for (int64_t s = 0; s < count; ++s) {
    if (s > 0) cursor_next<RPW>(a, cur_pos);
    const SliceRef cur = locate_slice<D, PAGED>(a, cur_pos, grp);
    issue_rows(a, cur, gl, buf);
    score(cur, buf);
  }
  publish_scores(a);
}

template <typename T, int D, int METHOD, bool PAGED>
static int launch_stream(ScoreDev& a, cudaStream_t st) {
  constexpr int RPW = 8 * (32 / (D / 8));
  auto kern = score_stream_kernel<T, D, METHOD, PAGED>;
  int occ = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, 0);
  if (occ < 1) occ = 1;
  a.slices_per_seg = (a.max_tokens + RPW - 1) / RPW;
  a.total_slices = (int64_t)a.batch * a.kv_heads * a.slices_per_seg;
  int64_t warps = (int64_t)num_sms() * occ * 8;
  if (warps > a.total_slices) warps = a.total_slices;
  a.slices_per_warp = (a.total_slices + warps - 1) / warps;
  const int64_t used_warps = (a.total_slices + a.slices_per_warp - 1) / a.slices_per_warp;
  const int blocks = (int)((used_warps + 7) / 8);
  kern<<<blocks, 256, 0, st>>>(a);
  return after_launch("mskv_score");
}

// Generic path: any head_dim, element-wise loads, one warp per row.
template <typename T, int METHOD>
__global__ void __launch_bounds__(256) score_generic_kernel(const ScoreDev a) {
  allow_dependents();  // the top-k kernel may become resident as this grid drains
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t nseg = (int64_t)a.batch * a.kv_heads;
  const int G = a.q_heads / a.kv_heads;
  const int64_t es = sizeof(T);
  for (int64_t r = warp; r < nseg * a.max_tokens; r += nwarps) {
    const int64_t seg = r / a.max_tokens;
    const int64_t t = r - seg * a.max_tokens;
    const int b = (int)(seg / a.kv_heads);
    const int h = (int)(seg - (int64_t)b * a.kv_heads);
    uint32_t why = 0;
    const int64_t off = rows_offset(a.k, b, h, t, &why, MSKV_STATUS_INDEX_OOB);
    if (off < 0) continue;  // beyond len[b] or unmapped page: nothing to score
    float acc = 0.f;
    for (int d = lane; d < a.head_dim; d += 32) {
      const float kv = load_f32<T>(a.k.base_k + off + d * es);
      if constexpr (METHOD == 0) {
        float qsum = 0.f;
        for (int g = 0; g < G; ++g)
          qsum += load_f32<T>(a.q + (int64_t)b * a.q_sb + (int64_t)(h * G + g) * a.q_sh + d * es);
        acc = fmaf(qsum, kv, acc);
      } else {
        acc = fmaf(kv, kv, acc);
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) put_score(a, seg * a.scores_stride + t, METHOD == 1 ? sqrtf(acc) : acc);
  }
  publish_scores(a);
}

template <typename T, int D, int METHOD, bool PAGED>
static int launch_fast(ScoreDev& a, cudaStream_t st) {
  auto kern = score_fast_kernel<T, D, METHOD, PAGED>;
  int occ = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, 0);
  if (occ < 1) occ = 1;
  a.slices_per_seg = (a.max_tokens + 31) / 32;
  a.total_slices = (int64_t)a.batch * a.kv_heads * a.slices_per_seg;
  int64_t warps = (int64_t)num_sms() * occ * 8;
  if (warps > a.total_slices) warps = a.total_slices;
  a.slices_per_warp = (a.total_slices + warps - 1) / warps;
  const int64_t used_warps = (a.total_slices + a.slices_per_warp - 1) / a.slices_per_warp;
  const int blocks = (int)((used_warps + 7) / 8);
  kern<<<blocks, 256, 0, st>>>(a);
  return after_launch("mskv_score");
}

template <typename T, int METHOD>
static int dispatch_d(ScoreDev& a, bool paged, bool fast, bool stream16, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    if (stream16) {
      if (a.head_dim == 64) return paged ? launch_stream<T, 64, METHOD, true>(a, st) : launch_stream<T, 64, METHOD, false>(a, st);
      if (a.head_dim == 128) return paged ? launch_stream<T, 128, METHOD, true>(a, st) : launch_stream<T, 128, METHOD, false>(a, st);
      if (a.head_dim == 256) return paged ? launch_stream<T, 256, METHOD, true>(a, st) : launch_stream<T, 256, METHOD, false>(a, st);
    }
  }
  if (fast) {
#define MSKV_SCORE_CASE(DD)                                                      \
  if (a.head_dim == DD) return paged ? launch_fast<T, DD, METHOD, true>(a, st)   \
                                     : launch_fast<T, DD, METHOD, false>(a, st);
    if constexpr (sizeof(T) == 2) {
      MSKV_SCORE_CASE(64)
      MSKV_SCORE_CASE(128)
      MSKV_SCORE_CASE(256)
    } else {
      MSKV_SCORE_CASE(32)
      MSKV_SCORE_CASE(64)
      MSKV_SCORE_CASE(128)
    }
#undef MSKV_SCORE_CASE
  }
  const int64_t rows = (int64_t)a.batch * a.kv_heads * a.max_tokens;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  score_generic_kernel<T, METHOD><<<(int)blocks, 256, 0, st>>>(a);
  return after_launch("mskv_score");
}

template <typename T>
static int dispatch_method(ScoreDev& a, bool paged, bool fast, bool stream16, cudaStream_t st) {
  return a.method == 0 ? dispatch_d<T, 0>(a, paged, fast, stream16, st) : dispatch_d<T, 1>(a, paged, fast, stream16, st);
}

}  // namespace mskv

using namespace mskv;

static int score_impl(const mskv_score_desc* d, float* const* peers, int npeers, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_score: NULL descriptor");
  if (d->batch < 0 || d->kv_heads <= 0 || d->q_heads <= 0 || d->head_dim <= 0 || d->max_tokens < 0)
    return fail(MSKV_ERR_ARG, "mskv_score: bad sizes");
  if (d->q_heads % d->kv_heads) return fail(MSKV_ERR_ARG, "mskv_score: q_heads %% kv_heads != 0");
  if (d->method != 0 && d->method != 1) return fail(MSKV_ERR_ARG, "mskv_score: method must be 0 or 1");
  if (!d->scores || (d->method == 0 && !d->q)) return fail(MSKV_ERR_ARG, "mskv_score: NULL q/scores");
  if (d->k.ring_start) return fail(MSKV_ERR_ARG, "mskv_score: ring-addressed keys are not supported");
  int rc = check_rows(d->k, "mskv_score k", false);
  if (rc) return rc;
  if (d->scores_stride < d->max_tokens) return fail(MSKV_ERR_ARG, "mskv_score: scores_stride < max_tokens");
  if (d->max_tokens > 0x7fffffffLL) return fail(MSKV_ERR_RANGE, "mskv_score: max_tokens exceeds 31 bits");
  if (d->batch == 0 || d->max_tokens == 0) return MSKV_OK;
  int es;
  switch (d->dtype) {
    case MSKV_DT_F32: es = 4; break;
    case MSKV_DT_F16: case MSKV_DT_BF16: es = 2; break;
    default: return fail(MSKV_ERR_DTYPE, "mskv_score: dtype must be f32, f16 or bf16");
  }
  ScoreDev a{};
  a.k = to_dev(d->k);
  a.q = static_cast<const char*>(d->q);
  a.q_sb = d->q_stride_b; a.q_sh = d->q_stride_h;
  a.scores = d->scores; a.scores_stride = d->scores_stride; a.max_tokens = d->max_tokens;
  a.batch = d->batch; a.q_heads = d->q_heads; a.kv_heads = d->kv_heads; a.head_dim = d->head_dim;
  a.method = d->method;
  a.npeers = npeers;
  for (int p = 0; p < npeers; ++p) a.peers[p] = peers[p];
  const bool paged = d->k.page_table != nullptr;
  a.page_shift = -1;
  if (paged && d->k.page_size > 0 && (d->k.page_size & (d->k.page_size - 1)) == 0) {
    int sh = 0;
    while ((1 << sh) < d->k.page_size) ++sh;
    a.page_shift = sh;
  }
  // The fast path needs 16-byte aligned rows/queries and, when paged, groups of up to 16
  // consecutive rows that never straddle a page.
  uint64_t al = (uint64_t)(uintptr_t)d->k.base_k | (uint64_t)d->k.stride_h | (uint64_t)d->k.stride_t;
  al |= paged ? (uint64_t)d->k.stride_page : (uint64_t)d->k.stride_b;
  if (d->method == 0) al |= (uint64_t)(uintptr_t)d->q | (uint64_t)d->q_stride_b | (uint64_t)d->q_stride_h;
  bool fast = (al & 15) == 0 && d->k.stride_t >= (int64_t)d->head_dim * es;
  if (paged) {
    const int epv = 16 / es;
    const int lpr = d->head_dim / epv;
    const int gl = lpr < 16 ? lpr : 16;
    fast = fast && gl > 0 && (d->k.page_size % gl) == 0;
  }
  // The 16-bit streaming path needs head_dim 64/128/256 and, when paged, pages holding whole
  // 8-row groups.
  bool stream16 = fast && es == 2 && (d->head_dim == 64 || d->head_dim == 128 || d->head_dim == 256);
  if (paged) stream16 = stream16 && (d->k.page_size % 8) == 0;
  cudaStream_t st = as_stream(stream);
  switch (d->dtype) {
    case MSKV_DT_F32: return dispatch_method<float>(a, paged, fast, false, st);
    case MSKV_DT_F16: return dispatch_method<__half>(a, paged, fast, stream16, st);
    default: return dispatch_method<__nv_bfloat16>(a, paged, fast, stream16, st);
  }
}

extern "C" int mskv_score(const mskv_score_desc* d, void* stream) { return score_impl(d, nullptr, 0, stream); }

extern "C" int mskv_score_fanout(const mskv_score_desc* d, float* const* peer_scores, int32_t npeers, void* stream) {
  if (npeers < 0 || npeers > kMaxPeers) return fail(MSKV_ERR_ARG, "mskv_score_fanout: npeers must lie in [0, %d]", kMaxPeers);
  if (npeers > 0 && !peer_scores) return fail(MSKV_ERR_ARG, "mskv_score_fanout: NULL peer_scores");
  for (int p = 0; p < npeers; ++p)
    if (!peer_scores[p]) return fail(MSKV_ERR_ARG, "mskv_score_fanout: NULL peer_scores[%d]", p);
  return score_impl(d, peer_scores, npeers, stream);
}
