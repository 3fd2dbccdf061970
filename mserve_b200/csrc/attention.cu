// Decode attention over the selected rows (mskv_sparse_attention).
//
// Reference: sparse_sdpa_attention (qwen-eljrte/Qwen_Transformer/attention.py:591-641):
// softmax(q·K_selᵀ/sqrt(D))·V_sel with no mask.  Here K_sel/V_sel keep the KV-head layout
// (no repeat_kv): all G query heads (times q_len query rows) of a KV head are served by one
// pass over that head's selected rows, so every gathered byte is read once from HBM.
//
// Split-sequence ("flash-decoding") schedule on the tensor cores, fast path (16-bit, D in
// {64,128}, G*q_len <= 16, 16-byte aligned rows): CTA (segment, split) owns kAtTile = 128
// selected rows, 32 per warp; see attn_mma_kernel.  The splits' (m, l, O) partials are merged
// by a second kernel, one block per (segment, query row).
// Other shapes use a one-warp-per-output-row kernel with an online softmax.
#include <math.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace mskv {
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
}  // namespace mskv

namespace mskv {

constexpr int kAtThreads = 128;
constexpr int kAtTile = 128;        // selected rows per CTA (32 per warp)

struct AttnDev {
  const char* q;
  int64_t q_sb, q_sh, q_sq;
  const char* k;
  const char* v;
  int64_t kv_seg, kv_s;
  const int32_t* counts;
  char* out;
  int64_t o_sb, o_sh, o_sq;
  float* ws;               // [segments][splits][nr][D + 2]
  uint32_t* status;
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

// Butterfly reduce-scatter of NV values over the M lanes of a group (lane bits below M):
// afterwards lane l holds in v[0 .. NV/M) the group sums of values [l*NV/M, (l+1)*NV/M).
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

// ---- tensor-core fragments (mma.sync m16n8k16, fp32 accumulate) -----------------------
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

// Fast path: the query rows of one KV head (G*q_len <= 16, padded to the MMA's 16 rows) against
// a tile of kAtTile selected rows.  Warp w owns rows [32w, 32w+32) of the tile:
//   * its K and V rows arrive as 16-byte cp.async chunks into shared memory with a padded row
//     stride (ROWB + 16 bytes, so ldmatrix reads are bank-conflict free);
//   * S = Q·Kᵀ: 4 n-tiles x D/16 k-steps of mma.m16n8k16 (K rows are the col-major B operand,
//     ldmatrix without transpose), fp32 accumulate; scale, mask rows beyond the count, row
//     max/sum across the four lanes that share a query row;
//   * O = P·V: P is re-packed from the S accumulators into A fragments (bf16/fp16), V comes
//     in through ldmatrix.trans; D/8 n-tiles x 2 k-steps;
//   * the four warps' (m, l, O) are merged in shared memory into the CTA's split partial in
//     the workspace; attn_merge_kernel then merges the splits and writes the output.
// The MMAs do not speed up a memory-bound step; they remove the per-element fp32 conversions
// and FMAs that made a CUDA-core version instruction bound.
template <bool BF16, int D>
__global__ void __launch_bounds__(kAtThreads) attn_mma_kernel(const AttnDev a) {
  allow_dependents();  // the split merge may become resident as this grid drains
  constexpr int ROWB = D * 2;
  constexpr int ROWP = ROWB + 16;       // padded shared-memory row stride (bytes)
  constexpr int KS = D / 16;            // k-steps of Q·Kᵀ
  constexpr int NT = D / 8;             // n-tiles of P·V
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem;                                   // [kAtTile][ROWP]
  uint8_t* sV = smem + kAtTile * ROWP;                  // [kAtTile][ROWP]
  uint8_t* sQ = smem + 2 * kAtTile * ROWP;              // [16][ROWP]
  __shared__ float s_m[4][16], s_l[4][16];

  const int seg = blockIdx.x / a.splits;
  const int split = blockIdx.x - seg * a.splits;
  const int b = seg / a.kv_heads;
  const int hk = seg - b * a.kv_heads;
  const int G = a.q_heads / a.kv_heads;
  const int nr = a.nr;
  int count = a.counts ? a.counts[seg] : a.num_sel;
  if (count > a.num_sel) count = a.num_sel;
  if (count < 0) count = 0;
  const int r0 = split * kAtTile;
  const int nrows = max(0, min(kAtTile, count - r0));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int wrow0 = warp * 32;                          // first tile row of this warp
  const int wrows = max(0, min(32, nrows - wrow0));     // this warp's valid rows

  // query rows (zero beyond nr), 16-byte chunks
  for (int x = tid; x < 16 * (ROWB / 16); x += kAtThreads) {
    const int r = x / (ROWB / 16), c = x - r * (ROWB / 16);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nr) {
      const int gq = r / a.q_len, i = r - gq * a.q_len;
      v = *reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.q_sb + (int64_t)(hk * G + gq) * a.q_sh +
                                          (int64_t)i * a.q_sq + c * 16);
    }
    *reinterpret_cast<uint4*>(sQ + r * ROWP + c * 16) = v;
  }
  // this warp's K/V rows: 16-byte cp.async chunks into the padded layout (a warp moves two
  // contiguous 256-byte rows per instruction); rows past the count are zero-filled so the
  // masked (P = 0) columns of P·V multiply finite values
  {
    constexpr int CPR = ROWB / 16;                       // chunks per row
    const char* kbase = a.k + (int64_t)seg * a.kv_seg + (int64_t)(r0 + wrow0) * a.kv_s;
    const char* vbase = a.v + (int64_t)seg * a.kv_seg + (int64_t)(r0 + wrow0) * a.kv_s;
    for (int x = lane; x < 32 * CPR; x += 32) {
      const int r = x / CPR, c = x - r * CPR;
      uint8_t* dk = sK + (wrow0 + r) * ROWP + c * 16;
      uint8_t* dv = sV + (wrow0 + r) * ROWP + c * 16;
      if (r < wrows) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dk)),
                     "l"(kbase + (int64_t)r * a.kv_s + c * 16) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dv)),
                     "l"(vbase + (int64_t)r * a.kv_s + c * 16) : "memory");
      } else {
        *reinterpret_cast<uint4*>(dk) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dv) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  __syncthreads();  // query rows visible to every warp
  // Q fragments for all k-steps (rows 0..15)
  uint32_t qa[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int col = kk * 16 + 8 * (lane >> 4);
    ldsm_x4(qa[kk], sQ + row * ROWP + col * 2);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();     // the warp's own rows (copied and zero-filled by its lanes) are visible

  // S = Q·Kᵀ for the warp's 32 rows: n-tile j covers rows wrow0 + 8j .. +7
  float sacc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) sacc[j][e] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int kk = 0; kk < KS; kk += 2) {
      uint32_t kb[4];
      const int row = wrow0 + 8 * j + (lane & 7);
      const int col = kk * 16 + 8 * (lane >> 3);
      ldsm_x4(kb, sK + row * ROWP + col * 2);
      mma16816<BF16>(sacc[j], qa[kk], kb[0], kb[1]);
      if (kk + 1 < KS) mma16816<BF16>(sacc[j], qa[kk + 1], kb[2], kb[3]);
    }
  }
  // scale, mask, row statistics (rows g and g+8; the four lanes of a group share a row)
  float m_lo = -INFINITY, m_hi = -INFINITY;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 8 * j + 2 * tig + (e & 1);
      const float v = col < wrows ? sacc[j][e] * a.scale : -INFINITY;
      sacc[j][e] = v;
      if (e < 2) m_lo = fmaxf(m_lo, v);
      else m_hi = fmaxf(m_hi, v);
    }
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    m_lo = fmaxf(m_lo, __shfl_xor_sync(0xffffffffu, m_lo, o));
    m_hi = fmaxf(m_hi, __shfl_xor_sync(0xffffffffu, m_hi, o));
  }
  float l_lo = 0.f, l_hi = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float mm = e < 2 ? m_lo : m_hi;
      const float p = (sacc[j][e] == -INFINITY) ? 0.f : __expf(sacc[j][e] - mm);
      sacc[j][e] = p;
      if (e < 2) l_lo += p;
      else l_hi += p;
    }
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, o);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, o);
  }
  // O = P·V: P as A fragments (two k-steps of 16 rows), V via ldmatrix.trans
  uint32_t pa[2][4];
#pragma unroll
  for (int k2 = 0; k2 < 2; ++k2) {
    pa[k2][0] = pack2<BF16>(sacc[2 * k2][0], sacc[2 * k2][1]);
    pa[k2][1] = pack2<BF16>(sacc[2 * k2][2], sacc[2 * k2][3]);
    pa[k2][2] = pack2<BF16>(sacc[2 * k2 + 1][0], sacc[2 * k2 + 1][1]);
    pa[k2][3] = pack2<BF16>(sacc[2 * k2 + 1][2], sacc[2 * k2 + 1][3]);
  }
  float oacc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) oacc[n][e] = 0.f;
#pragma unroll
  for (int k2 = 0; k2 < 2; ++k2) {
#pragma unroll
    for (int n = 0; n < NT; n += 2) {
      uint32_t vb[4];
      const int row = wrow0 + 16 * k2 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int col = n * 8 + 8 * (lane >> 4);
      ldsm_x4_t(vb, sV + row * ROWP + col * 2);
      mma16816<BF16>(oacc[n], pa[k2], vb[0], vb[1]);
      mma16816<BF16>(oacc[n + 1], pa[k2], vb[2], vb[3]);
    }
  }
  // warp partial -> shared memory (the warp's own K rows are free now): O as fp32 [16][OS],
  // row stride OS = D + 8 floats so each half-warp's 8-byte stores hit 32 distinct banks;
  // 16 * OS * 4 bytes == 32 * ROWP, exactly the warp's rows
  constexpr int OS = D + 8;
  static_assert(16 * OS * 4 <= 32 * ROWP, "warp partial must fit in the warp's K rows");
  __syncwarp();
  float* so = reinterpret_cast<float*>(sK + wrow0 * ROWP);
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int col = n * 8 + 2 * tig;
    *reinterpret_cast<float2*>(so + g * OS + col) = make_float2(oacc[n][0], oacc[n][1]);
    *reinterpret_cast<float2*>(so + (g + 8) * OS + col) = make_float2(oacc[n][2], oacc[n][3]);
  }
  if (tig == 0) {
    s_m[warp][g] = wrows > 0 ? m_lo : -INFINITY;
    s_m[warp][g + 8] = wrows > 0 ? m_hi : -INFINITY;
    s_l[warp][g] = l_lo;
    s_l[warp][g + 8] = l_hi;
  }
  __syncthreads();
  // merge the four warps -> this CTA's split partial
  const int64_t wstride = (int64_t)a.nr * (D + 2);
  float* wp = a.ws + ((int64_t)seg * a.splits + split) * wstride;
  for (int x = tid; x < nr * D; x += kAtThreads) {
    const int r = x / D, d = x - r * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][r]);
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (s_m[w][r] == -INFINITY) continue;
      const float f = __expf(s_m[w][r] - M);
      L += s_l[w][r] * f;
      o += reinterpret_cast<const float*>(sK + w * 32 * ROWP)[r * OS + d] * f;
    }
    wp[(int64_t)r * (D + 2) + d] = o;
    if (d == 0) {
      wp[(int64_t)r * (D + 2) + D] = M;
      wp[(int64_t)r * (D + 2) + D + 1] = L;
    }
  }
}

// Merges the split partials of one (segment, query row) per block (one thread per output dim):
// every split's maximum, normaliser and value are independent loads, so the merge costs about
// one L2 round trip.
template <typename T, int D>
__global__ void __launch_bounds__(D) attn_merge_kernel(const AttnDev a) {
  wait_for_previous_grid();  // the split partials come from attn_mma_kernel (programmatic launch)
  const int seg = blockIdx.x / a.nr, r = blockIdx.x - (blockIdx.x / a.nr) * a.nr;
  const int d = threadIdx.x;
  const int64_t wstride = (int64_t)a.nr * (D + 2);
  const float* rb = a.ws + (int64_t)seg * a.splits * wstride + (int64_t)r * (D + 2);
  float M = -INFINITY;
#pragma unroll 8
  for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, rb[sp * wstride + D]);
  float L = 0.f, o = 0.f;
#pragma unroll 8
  for (int sp = 0; sp < a.splits; ++sp) {
    const float ms = rb[sp * wstride + D];
    const float w = ms == -INFINITY ? 0.f : __expf(ms - M);
    L += rb[sp * wstride + D + 1] * w;
    o += rb[sp * wstride + d] * w;
  }
  const int b = seg / a.kv_heads, hk = seg - b * a.kv_heads;
  const int G = a.q_heads / a.kv_heads;
  const int gq = r / a.q_len, i = r - gq * a.q_len;
  T* op = reinterpret_cast<T*>(a.out + (int64_t)b * a.o_sb + (int64_t)(hk * G + gq) * a.o_sh + (int64_t)i * a.o_sq);
  op[d] = from_f<T>(L > 0.f ? o / L : 0.f);
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

static int dtype_size(int dt) {
  switch (dt) {
    case MSKV_DT_F32: return 4;
    case MSKV_DT_F16: case MSKV_DT_BF16: return 2;
    default: return 0;
  }
}

static bool fast_path(const mskv_attn_desc* d) {
  if (dtype_size(d->dtype) != 2) return false;
  if (d->head_dim != 64 && d->head_dim != 128) return false;
  const int G = d->q_heads / d->kv_heads;
  if (G * d->q_len > 16) return false;                            // one m16 MMA row block
  // the split merge keeps one weight per (split, query row) in the V tile's shared memory
  const int64_t splits = d->num_selected > 0 ? (d->num_selected + kAtTile - 1) / kAtTile : 1;
  if ((splits + 1) * 16 * 4 > (int64_t)kAtTile * (d->head_dim * 2 + 16)) return false;
  const uint64_t al = (uint64_t)(uintptr_t)d->k | (uint64_t)(uintptr_t)d->v | (uint64_t)d->kv_stride_seg |
                      (uint64_t)d->kv_stride_s | (uint64_t)(uintptr_t)d->q | (uint64_t)d->q_stride_b |
                      (uint64_t)d->q_stride_h | (uint64_t)d->q_stride_q;
  return (al & 15) == 0;                                          // 16-byte bulk copies / loads
}

static int64_t splits_of(const mskv_attn_desc* d) {
  return d->num_selected > 0 ? (d->num_selected + kAtTile - 1) / kAtTile : 1;
}

}  // namespace mskv

using namespace mskv;

extern "C" uint64_t mskv_attention_workspace_bytes(const mskv_attn_desc* d) {
  if (!d || d->kv_heads <= 0 || d->q_heads <= 0 || d->q_len <= 0 || d->batch < 0) return 0;
  if (!fast_path(d)) return 0;
  const int64_t nr = (int64_t)(d->q_heads / d->kv_heads) * d->q_len;
  return (uint64_t)((int64_t)d->batch * d->kv_heads * splits_of(d) * nr * (d->head_dim + 2) * 4);
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
  a.status = d->status;
  a.scale = d->scale; a.batch = d->batch; a.q_heads = d->q_heads; a.kv_heads = d->kv_heads;
  a.head_dim = d->head_dim; a.q_len = d->q_len; a.num_sel = d->num_selected; a.dtype = d->dtype;
  a.nr = (d->q_heads / d->kv_heads) * d->q_len;
  cudaStream_t st = as_stream(stream);
  if (fast_path(d)) {
    const uint64_t need = mskv_attention_workspace_bytes(d);
    if (!d->workspace || d->workspace_bytes < need)
      return fail(MSKV_ERR_ARG, "mskv_sparse_attention: workspace needs %llu bytes", (unsigned long long)need);
    if (((uintptr_t)d->workspace & 255) != 0) return fail(MSKV_ERR_ARG, "mskv_sparse_attention: workspace must be 256-byte aligned");
    a.ws = static_cast<float*>(d->workspace);
    a.splits = (int)splits_of(d);
    const int64_t blocks = (int64_t)d->batch * d->kv_heads * a.splits;
    if (blocks > 0x7fffffffLL) return fail(MSKV_ERR_RANGE, "mskv_sparse_attention: grid too large");
    const bool bf = d->dtype == MSKV_DT_BF16;
    const int smem = (2 * kAtTile + 16) * (d->head_dim * 2 + 16);
    const void* kern = d->head_dim == 128 ? (bf ? (const void*)attn_mma_kernel<true, 128> : (const void*)attn_mma_kernel<false, 128>)
                                          : (bf ? (const void*)attn_mma_kernel<true, 64> : (const void*)attn_mma_kernel<false, 64>);
    int rc0 = ensure_smem_limit(kern, 80 * 1024, "mskv_sparse_attention");
    if (rc0) return rc0;
    if (d->head_dim == 128) {
      if (bf) attn_mma_kernel<true, 128><<<(unsigned)blocks, kAtThreads, smem, st>>>(a);
      else attn_mma_kernel<false, 128><<<(unsigned)blocks, kAtThreads, smem, st>>>(a);
    } else {
      if (bf) attn_mma_kernel<true, 64><<<(unsigned)blocks, kAtThreads, smem, st>>>(a);
      else attn_mma_kernel<false, 64><<<(unsigned)blocks, kAtThreads, smem, st>>>(a);
    }
    int rc = after_launch("mskv_sparse_attention");
    if (rc) return rc;
    const unsigned mblocks = (unsigned)((int64_t)d->batch * d->kv_heads * a.nr);
    cudaError_t e;
    if (d->head_dim == 128) {
      e = bf ? launch_dependent(attn_merge_kernel<__nv_bfloat16, 128>, dim3(mblocks), dim3(128), 0, st, a)
             : launch_dependent(attn_merge_kernel<__half, 128>, dim3(mblocks), dim3(128), 0, st, a);
    } else {
      e = bf ? launch_dependent(attn_merge_kernel<__nv_bfloat16, 64>, dim3(mblocks), dim3(64), 0, st, a)
             : launch_dependent(attn_merge_kernel<__half, 64>, dim3(mblocks), dim3(64), 0, st, a);
    }
    if (e != cudaSuccess) return cuda_status(e, "mskv_sparse_attention merge launch");
    return after_launch("mskv_sparse_attention");
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

// ---------------------------------------------------------------------------------------
// Allocation-free variant of mskv_sparse_attention.
//
// Some callers cannot allocate device memory at the point where they run attention: code
// that runs under an allocator lock or inside another library's memory pool, plugins whose
// host framework forbids cudaMalloc on its hot path, or callers that have no allocator of
// their own to hand out a workspace.  For them the split-sequence workspace lives in one
// file-scope device array of MSKV_NOALLOC_ATTN_SCRATCH_BYTES, which every GPU that loads
// this library keeps until the process exits.  Its device address is looked up once per
// device (cudaGetSymbolAddress, on that device's first call) and cached together with the id
// of the CUDA context it belongs to; a call from another context of that device (after a
// cudaDeviceReset, or once the primary context was released and created again) looks the
// address up again.  Nothing is allocated or freed.  Each call rewrites every partial it later
// reads, so nothing in the array has to start at zero; but all calls on a device share it, so
// calls that overlap on the GPU (different streams without ordering) race on it.
static __device__ __align__(256) unsigned char g_attn_scratch[MSKV_NOALLOC_ATTN_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
struct ScratchAddr {
  void* ptr;
  unsigned long long ctx_id;   // 0: not looked up yet
};
std::mutex g_scratch_mu;
ScratchAddr g_scratch_dev[kMaxDevices] = {};

// Id of the calling thread's current CUDA context (driver API through the runtime's entry
// point, so the library links only the runtime); 0 when there is none yet.
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(f);
    cudaGetLastError();
  });
  if (!get_current || !get_id) return 0;
  void* ctx = nullptr;
  if (get_current(&ctx) != 0 || !ctx) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == 0 ? id : 0;
}

int scratch_of_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MSKV_ERR_RANGE, "device index %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& c = g_scratch_dev[dev];
  const unsigned long long id = current_context_id();
  if (!c.ptr || id == 0 || c.ctx_id != id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);   // also creates the context if needed
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(attention scratch)");
    c.ptr = p;
    c.ctx_id = current_context_id();
  }
  *out = c.ptr;
  return MSKV_OK;
}
}  // namespace

extern "C" int mskv_sparse_attention_noalloc(const mskv_attn_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_sparse_attention_noalloc: NULL descriptor");
  const uint64_t need = mskv_attention_workspace_bytes(d);
  if (need > (uint64_t)MSKV_NOALLOC_ATTN_SCRATCH_BYTES)
    return fail(MSKV_ERR_RANGE,
                "mskv_sparse_attention_noalloc: this shape needs %llu bytes of scratch, more than the built-in "
                "%llu; use mskv_sparse_attention with a caller-provided workspace",
                (unsigned long long)need, (unsigned long long)MSKV_NOALLOC_ATTN_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = scratch_of_current_device(&scratch);
  if (rc != MSKV_OK) return rc;
  mskv_attn_desc c = *d;
  c.workspace = scratch;
  c.workspace_bytes = MSKV_NOALLOC_ATTN_SCRATCH_BYTES;
  return mskv_sparse_attention(&c, stream);
}
