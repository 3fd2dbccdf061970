// Decode attention over the selected rows (mskv_sparse_attention).
//
// Reference: sparse_sdpa_attention (qwen-eljrte/Qwen_Transformer/attention.py:591-641):
// softmax(q·K_selᵀ/sqrt(D))·V_sel with no mask.  Here K_sel/V_sel keep the KV-head layout
// (no repeat_kv): all G query heads (times q_len query rows) of a KV head are served by one
// pass over that head's selected rows, so every gathered byte is read once from HBM.
//
// Split-sequence ("flash-decoding") schedule: CTA (segment, split) handles kTile rows.
//   1. each 16-lane group loads 16 K rows (one 16-byte chunk per lane per row), converts
//      once to fp32, and for every query row reduce-scatters the 16 partial dot products
//      so lane l ends with the score of row l -> shared memory;
//   2. per query row: tile max, exp, sum (fp32);
//   3. V rows are streamed the same way and accumulated into per-lane fp32 accumulators,
//      merged across groups with shared-memory atomics;
//   4. (m, l, acc[D]) partials go to the workspace; a combine kernel merges the splits and
//      writes the output in the input dtype.
// Shapes outside the fast path (head_dim != 64/128, 32-bit types, > 8 query rows per KV
// head) use a one-warp-per-output-row kernel with an online softmax.
#include <math.h>

#include "common.cuh"

namespace mskv {

constexpr int kAtThreads = 256;
constexpr int kTile = 256;      // rows per CTA
constexpr int kMaxNR = 8;       // query rows per KV head on the fast path

struct AttnDev {
  const char* q;
  int64_t q_sb, q_sh, q_sq;
  const char* k;
  const char* v;
  int64_t kv_seg, kv_s;
  const int32_t* counts;
  char* out;
  int64_t o_sb, o_sh, o_sq;
  float* ws;               // [seg][split][NR][D + 2]
  float scale;
  int32_t batch, q_heads, kv_heads, head_dim, q_len, num_sel, splits, nr, dtype;
};

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ void cvt8(const uint4& v, float* f, bool is_bf16) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (is_bf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      __half2 h;
      memcpy(&h, &w[i], 4);
      const float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
}

template <int N>
__device__ __forceinline__ float reduce_scatter_a(float (&v)[N], int lane) {
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

// Fast path: 16-bit types, D in {64, 128}; GL = D/8 lanes per row (8 or 16).
template <bool BF16, int D>
__global__ void __launch_bounds__(kAtThreads, 1) attn_partial_kernel(const AttnDev a) {
  constexpr int GL = D / 8;                  // lanes per row == rows per group iteration
  __shared__ float s_q[kMaxNR][D];
  __shared__ float s_p[kMaxNR][kTile];
  __shared__ float s_acc[kMaxNR][D];
  __shared__ float s_m[kMaxNR], s_l[kMaxNR];

  const int seg = blockIdx.x / a.splits;
  const int split = blockIdx.x - seg * a.splits;
  const int b = seg / a.kv_heads;
  const int hk = seg - b * a.kv_heads;
  const int G = a.q_heads / a.kv_heads;
  const int nr = a.nr;
  int count = a.counts ? a.counts[seg] : a.num_sel;
  if (count > a.num_sel) count = a.num_sel;
  if (count < 0) count = 0;
  const int r0 = split * kTile;
  const int nrows = max(0, min(kTile, count - r0));

  // Query rows of this KV head (row r = g*q_len + i) -> fp32 shared memory, pre-scaled.
  for (int x = threadIdx.x; x < nr * D; x += kAtThreads) {
    const int r = x / D, d = x - r * D;
    const int g = r / a.q_len, i = r - g * a.q_len;
    const char* qp = a.q + (int64_t)b * a.q_sb + (int64_t)(hk * G + g) * a.q_sh + (int64_t)i * a.q_sq;
    const float qv = BF16 ? to_f(reinterpret_cast<const __nv_bfloat16*>(qp)[d])
                          : to_f(reinterpret_cast<const __half*>(qp)[d]);
    s_q[r][d] = qv * a.scale;
    s_acc[r][d] = 0.f;
  }
  __syncthreads();

  const int tid = threadIdx.x;
  const int gl = tid & (GL - 1);
  const char* kseg = a.k + (int64_t)seg * a.kv_seg;
  const char* vseg = a.v + (int64_t)seg * a.kv_seg;

  // Loops run per warp (uniform trip counts, so the shuffles see all 32 lanes); the
  // 32/GL groups of a warp take consecutive GL-row blocks of the warp's 32 rows.
  const int warp_id = tid >> 5;
  const int grp_in_warp = (tid & 31) / GL;
  // 1. scores
  for (int wb = warp_id * 32; wb < nrows; wb += kAtThreads) {
    const int rb = wb + grp_in_warp * GL;
    float f[GL][8];
#pragma unroll
    for (int j = 0; j < GL; ++j) {
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (rb + j < nrows)
        raw = *reinterpret_cast<const uint4*>(kseg + (int64_t)(r0 + rb + j) * a.kv_s + gl * 16);
      cvt8(raw, f[j], BF16);
    }
    for (int r = 0; r < nr; ++r) {
      float qf[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) qf[e] = s_q[r][gl * 8 + e];
      float part[GL];
#pragma unroll
      for (int j = 0; j < GL; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(qf[e], f[j][e], acc);
        part[j] = acc;
      }
      const float sc = reduce_scatter_a<GL>(part, gl);
      if (rb + gl < nrows) s_p[r][rb + gl] = sc;
    }
  }
  __syncthreads();

  // 2. tile softmax statistics: warp w handles query rows w, w+8, ...
  const int lane = tid & 31, warp = tid >> 5;
  for (int r = warp; r < nr; r += kAtThreads / 32) {
    float m = -INFINITY;
    for (int x = lane; x < nrows; x += 32) m = fmaxf(m, s_p[r][x]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int x = lane; x < nrows; x += 32) {
      const float p = expf(s_p[r][x] - m);
      s_p[r][x] = p;
      l += p;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) { s_m[r] = m; s_l[r] = l; }
  }
  __syncthreads();

  // 3. P·V
  float acc[kMaxNR][8];
#pragma unroll
  for (int r = 0; r < kMaxNR; ++r)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
  for (int wb = warp_id * 32; wb < nrows; wb += kAtThreads) {
    const int rb = wb + grp_in_warp * GL;
    uint4 raw[GL];
#pragma unroll
    for (int j = 0; j < GL; ++j) {
      raw[j] = make_uint4(0, 0, 0, 0);
      if (rb + j < nrows)
        raw[j] = *reinterpret_cast<const uint4*>(vseg + (int64_t)(r0 + rb + j) * a.kv_s + gl * 16);
    }
#pragma unroll
    for (int j = 0; j < GL; ++j) {
      if (rb + j < nrows) {
        float vf[8];
        cvt8(raw[j], vf, BF16);
#pragma unroll
        for (int r = 0; r < kMaxNR; ++r) {
          if (r < nr) {
            const float p = s_p[r][rb + j];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r][e] = fmaf(p, vf[e], acc[r][e]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kMaxNR; ++r)
    if (r < nr)
#pragma unroll
      for (int e = 0; e < 8; ++e) atomicAdd(&s_acc[r][gl * 8 + e], acc[r][e]);
  __syncthreads();

  // 4. partials
  float* wsp = a.ws + ((int64_t)seg * a.splits + split) * nr * (D + 2);
  for (int x = tid; x < nr * D; x += kAtThreads) {
    const int r = x / D, d = x - r * D;
    wsp[(int64_t)r * (D + 2) + d] = s_acc[r][d];
  }
  if (tid < nr) {
    wsp[(int64_t)tid * (D + 2) + D] = nrows > 0 ? s_m[tid] : -INFINITY;
    wsp[(int64_t)tid * (D + 2) + D + 1] = nrows > 0 ? s_l[tid] : 0.f;
  }
}

// Merges the splits of one (segment, query row) per warp and writes the output row.
template <typename T>
__global__ void attn_combine_kernel(const AttnDev a) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nseg = (int64_t)a.batch * a.kv_heads;
  if (wid >= nseg * a.nr) return;
  const int seg = (int)(wid / a.nr);
  const int r = (int)(wid - (int64_t)seg * a.nr);
  const int D = a.head_dim;
  const float* base = a.ws + (int64_t)seg * a.splits * a.nr * (D + 2) + (int64_t)r * (D + 2);
  const int64_t sstride = (int64_t)a.nr * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, base[s * sstride + D]);
  float L = 0.f;
  for (int s = 0; s < a.splits; ++s) {
    const float m = base[s * sstride + D];
    if (m != -INFINITY) L += base[s * sstride + D + 1] * expf(m - M);
  }
  const int b = seg / a.kv_heads, hk = seg - b * a.kv_heads;
  const int G = a.q_heads / a.kv_heads;
  const int g = r / a.q_len, i = r - g * a.q_len;
  T* op = reinterpret_cast<T*>(a.out + (int64_t)b * a.o_sb + (int64_t)(hk * G + g) * a.o_sh + (int64_t)i * a.o_sq);
  for (int d = lane; d < D; d += 32) {
    float o = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float m = base[s * sstride + D];
      if (m != -INFINITY) o += base[s * sstride + d] * expf(m - M);
    }
    op[d] = from_f<T>(L > 0.f ? o / L : 0.f);
  }
}

// Generic path: one warp per output row (b, hq, i); online softmax over the selected rows.
template <typename T>
__global__ void attn_generic_kernel(const AttnDev a) {
  constexpr int kMaxPerLane = 32;  // head_dim <= 1024
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)a.batch * a.q_heads * a.q_len;
  if (wid >= rows) return;
  const int i = (int)(wid % a.q_len);
  const int hq = (int)((wid / a.q_len) % a.q_heads);
  const int b = (int)(wid / ((int64_t)a.q_len * a.q_heads));
  const int G = a.q_heads / a.kv_heads;
  const int hk = hq / G;
  const int seg = b * a.kv_heads + hk;
  const int D = a.head_dim;
  int count = a.counts ? a.counts[seg] : a.num_sel;
  if (count > a.num_sel) count = a.num_sel;
  const T* qp = reinterpret_cast<const T*>(a.q + (int64_t)b * a.q_sb + (int64_t)hq * a.q_sh + (int64_t)i * a.q_sq);
  float qv[kMaxPerLane], acc[kMaxPerLane];
#pragma unroll
  for (int x = 0; x < kMaxPerLane; ++x) {
    const int d = lane + 32 * x;
    qv[x] = d < D ? to_f<T>(qp[d]) * a.scale : 0.f;
    acc[x] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int s = 0; s < count; ++s) {
    const T* kr = reinterpret_cast<const T*>(a.k + (int64_t)seg * a.kv_seg + (int64_t)s * a.kv_s);
    const T* vr = reinterpret_cast<const T*>(a.v + (int64_t)seg * a.kv_seg + (int64_t)s * a.kv_s);
    float dot = 0.f;
#pragma unroll
    for (int x = 0; x < kMaxPerLane; ++x) {
      const int d = lane + 32 * x;
      if (d < D) dot = fmaf(qv[x], to_f<T>(kr[d]), dot);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float mn = fmaxf(m, dot);
    const float corr = expf(m - mn);
    const float p = expf(dot - mn);
    l = l * corr + p;
#pragma unroll
    for (int x = 0; x < kMaxPerLane; ++x) {
      const int d = lane + 32 * x;
      if (d < D) acc[x] = acc[x] * corr + p * to_f<T>(vr[d]);
    }
    m = mn;
  }
  T* op = reinterpret_cast<T*>(a.out + (int64_t)b * a.o_sb + (int64_t)hq * a.o_sh + (int64_t)i * a.o_sq);
#pragma unroll
  for (int x = 0; x < kMaxPerLane; ++x) {
    const int d = lane + 32 * x;
    if (d < D) op[d] = from_f<T>(l > 0.f ? acc[x] / l : 0.f);
  }
}

static bool fast_path(const mskv_attn_desc* d, int es) {
  if (es != 2) return false;
  if (d->head_dim != 64 && d->head_dim != 128) return false;
  const int G = d->q_heads / d->kv_heads;
  if (G * d->q_len > kMaxNR) return false;
  const uint64_t al = (uint64_t)(uintptr_t)d->k | (uint64_t)(uintptr_t)d->v | (uint64_t)d->kv_stride_seg |
                      (uint64_t)d->kv_stride_s;
  return (al & 15) == 0;
}

static int dtype_size(int dt) {
  switch (dt) {
    case MSKV_DT_F32: return 4;
    case MSKV_DT_F16: case MSKV_DT_BF16: return 2;
    default: return 0;
  }
}

}  // namespace mskv

using namespace mskv;

extern "C" uint64_t mskv_attention_workspace_bytes(const mskv_attn_desc* d) {
  if (!d || d->kv_heads <= 0 || d->q_heads <= 0 || d->q_len <= 0 || d->batch < 0) return 0;
  const int es = dtype_size(d->dtype);
  if (!fast_path(d, es)) return 0;
  const int64_t splits = d->num_selected > 0 ? (d->num_selected + kTile - 1) / kTile : 1;
  const int64_t nr = (int64_t)(d->q_heads / d->kv_heads) * d->q_len;
  return (uint64_t)((int64_t)d->batch * d->kv_heads * splits * nr * (d->head_dim + 2) * 4);
}

extern "C" int mskv_sparse_attention(const mskv_attn_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_sparse_attention: NULL descriptor");
  if (d->batch < 0 || d->kv_heads <= 0 || d->q_heads <= 0 || d->head_dim <= 0 || d->q_len <= 0 ||
      d->num_selected < 0)
    return fail(MSKV_ERR_ARG, "mskv_sparse_attention: bad sizes");
  if (d->q_heads % d->kv_heads) return fail(MSKV_ERR_ARG, "mskv_sparse_attention: q_heads %% kv_heads != 0");
  if (d->head_dim > 1024) return fail(MSKV_ERR_RANGE, "mskv_sparse_attention: head_dim > 1024");
  const int es = dtype_size(d->dtype);
  if (!es) return fail(MSKV_ERR_DTYPE, "mskv_sparse_attention: dtype must be f32, f16 or bf16");
  if (!d->q || !d->out || (d->num_selected > 0 && (!d->k || !d->v)))
    return fail(MSKV_ERR_ARG, "mskv_sparse_attention: NULL pointer");
  if (d->batch == 0) return MSKV_OK;
  AttnDev a{};
  a.q = static_cast<const char*>(d->q); a.q_sb = d->q_stride_b; a.q_sh = d->q_stride_h; a.q_sq = d->q_stride_q;
  a.k = static_cast<const char*>(d->k); a.v = static_cast<const char*>(d->v);
  a.kv_seg = d->kv_stride_seg; a.kv_s = d->kv_stride_s; a.counts = d->counts;
  a.out = static_cast<char*>(d->out); a.o_sb = d->out_stride_b; a.o_sh = d->out_stride_h; a.o_sq = d->out_stride_q;
  a.scale = d->scale; a.batch = d->batch; a.q_heads = d->q_heads; a.kv_heads = d->kv_heads;
  a.head_dim = d->head_dim; a.q_len = d->q_len; a.num_sel = d->num_selected; a.dtype = d->dtype;
  a.nr = (d->q_heads / d->kv_heads) * d->q_len;
  cudaStream_t st = as_stream(stream);
  if (fast_path(d, es)) {
    const uint64_t need = mskv_attention_workspace_bytes(d);
    if (!d->workspace || d->workspace_bytes < need)
      return fail(MSKV_ERR_ARG, "mskv_sparse_attention: workspace needs %llu bytes", (unsigned long long)need);
    a.ws = static_cast<float*>(d->workspace);
    a.splits = d->num_selected > 0 ? (d->num_selected + kTile - 1) / kTile : 1;
    const int64_t blocks = (int64_t)d->batch * d->kv_heads * a.splits;
    const bool bf = d->dtype == MSKV_DT_BF16;
    if (d->head_dim == 128) {
      if (bf) attn_partial_kernel<true, 128><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
      else attn_partial_kernel<false, 128><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
    } else {
      if (bf) attn_partial_kernel<true, 64><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
      else attn_partial_kernel<false, 64><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
    }
    int rc = after_launch("mskv_sparse_attention partial");
    if (rc) return rc;
    const int64_t warps = (int64_t)d->batch * d->kv_heads * a.nr;
    const unsigned cblocks = (unsigned)((warps * 32 + 255) / 256);
    if (bf) attn_combine_kernel<__nv_bfloat16><<<cblocks, 256, 0, st>>>(a);
    else attn_combine_kernel<__half><<<cblocks, 256, 0, st>>>(a);
    return after_launch("mskv_sparse_attention combine");
  }
  const int64_t rows = (int64_t)d->batch * d->q_heads * d->q_len;
  const unsigned blocks = (unsigned)((rows * 32 + 255) / 256);
  switch (d->dtype) {
    case MSKV_DT_F32: attn_generic_kernel<float><<<blocks, 256, 0, st>>>(a); break;
    case MSKV_DT_F16: attn_generic_kernel<__half><<<blocks, 256, 0, st>>>(a); break;
    default: attn_generic_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a); break;
  }
  return after_launch("mskv_sparse_attention");
}
