// Decode attention over the selected rows (mskv_sparse_attention).
//
// Reference: sparse_sdpa_attention (qwen-eljrte/Qwen_Transformer/attention.py:591-641):
// softmax(q·K_selᵀ/sqrt(D))·V_sel with no mask.  Here K_sel/V_sel keep the KV-head layout
// (no repeat_kv): all G query heads (times q_len query rows) of a KV head are served by one
// pass over that head's selected rows, so every gathered byte is read once from HBM.
//
// Fast path (16-bit, D in {64,128}, G*q_len <= 16, 16-byte aligned rows and strides), on the
// tensor cores (mma.sync m16n8k16, fp32 accumulate):
//  * selections of up to 8 x 4096 rows: one streaming kernel, the CTAs of a segment forming a
//    thread-block cluster that merges through distributed shared memory (attn_cluster_kernel;
//    TMA tile loads, no workspace);
//  * wider selections: split-sequence ("flash-decoding") schedule, CTA (segment, split) owns
//    kAtTile = 128 rows (attn_mma_kernel), the splits' (m, l, O) partials in a workspace merged
//    by a second kernel, one block per (segment, query row).
// Other shapes use a one-warp-per-output-row kernel with an online softmax.
#include <cuda.h>   // CUtensorMap and its enums; the encoder is reached through the runtime
#include <math.h>

#include <algorithm>
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
  int32_t rps;             // streaming cluster path: selected rows per CTA (splits = CTAs per cluster)
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

// ---- streaming cluster path ------------------------------------------------------------
// One kernel per call, no workspace.  The CTAs of a segment (a (sequence, KV head) pair) form
// a thread-block cluster of cs <= 8; CTA c owns the selected rows [c*rps, (c+1)*rps), where cs
// and rps depend only on the selection width (so a segment is split the same way whatever the
// batch, the chunking or the head sharding of the call, and outputs are bit-identical across
// them).  Inside a CTA every warp streams its own 16-row blocks (blocks warp, warp+4, ...)
// through a private ring of kAcStages stages: one elected lane issues the block's K and V as
// tiled TMA loads (3-D tensor maps [segment][row][dim], 128-byte boxes with the 128-byte
// swizzle, so ldmatrix reads are bank-conflict free without padding) that complete on the
// stage's mbarrier, and refills the stage as soon as the warp has read it.  Rows past the
// selection width arrive zero-filled by the TMA unit; V rows between the segment's count and
// the width are zeroed in shared memory, so the masked (P = 0) columns of P·V stay finite.
// Each warp keeps an online softmax (running max, normaliser, O) in registers; the four warps
// merge in shared memory into the CTA's partial, and the cluster merges its CTAs' partials
// through distributed shared memory and writes the output.  Every mbarrier wait is bounded:
// past the limit the warp sets MSKV_STATUS_TIMEOUT, waits (bounded) for its other loads in
// flight, drops its rows and still takes every barrier, so the CTA and the cluster finish.
constexpr int kAcWarps = 4;
constexpr int kAcStages = 3;          // per warp
constexpr int kAcBlock = 16;          // selected rows per block (one k-step of P·V)
constexpr int kAcMaxCluster = 8;      // portable cluster size
constexpr int kAcRowsPerCta = 256;    // split target: cs = ceil(width / 256), at most 8
constexpr int kAcMaxWidth = kAcMaxCluster * 4096;   // wider selections take the split path
constexpr int kAcWaitIters = 1 << 22;

template <int D>
struct AcShape {
  static constexpr int HALVES = D / 64;                    // 128-byte column boxes per row
  static constexpr int HB = kAcBlock * 128;                // one box: 16 rows x 128 bytes
  static constexpr int KB = HALVES * HB;                   // K (or V) bytes of a block
  static constexpr int SB = 2 * KB;                        // stage: K block then V block
  static constexpr int ROWP = D * 2 + 16;                  // padded query row (bytes)
  static constexpr int SMEM = kAcWarps * kAcStages * SB + 16 * ROWP + 1024;   // + alignment slack
};

__device__ __forceinline__ bool ac_wait(uint32_t bar, uint32_t parity) {
  for (int it = 0; it < kAcWaitIters; ++it) {
    uint32_t done;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void ac_tma_load(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
               ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar) : "memory");
}

// Transpose of an 8x8 matrix of 16-bit values held one row-pair per thread (the mma.sync
// C/A fragment layout): thread (g, tig) receives elements (2 tig, g) and (2 tig + 1, g).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// 2^x by the SFU (ex2.approx.ftz: relative error about 2^-22; 2^-inf = 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(remote)
               : "memory");
  return v;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Byte offset of 16-byte chunk c (of a row of D/8 chunks) of block row `row` in a block stored
// as 128-byte-swizzled boxes of 16 rows x 128 bytes (chunk (c & 7) of box (c >> 3) sits at
// position (c & 7) ^ (row & 7) of its 128-byte line).
__device__ __forceinline__ int ac_swz(int row, int c) {
  return (c >> 3) * (kAcBlock * 128) + row * 128 + (((c & 7) ^ (row & 7)) << 4);
}

template <bool BF16, int D, bool NARROW>
__global__ void __launch_bounds__(kAcWarps * 32, 2)
    attn_cluster_kernel(const AttnDev a, const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv) {
  allow_dependents();
  using SH = AcShape<D>;
  constexpr int KS = D / 16;            // k-steps of Q·Kᵀ
  constexpr int NT = D / 8;             // n-tiles of P·V
  constexpr int OS = D + 8;             // padded row of a warp's fp32 partial
  static_assert(16 * OS * 4 <= 2 * SH::SB, "a warp's partial must fit in two of its stages");
  static_assert(16 * D * 4 <= SH::SB, "the CTA partial must fit in one stage");
  extern __shared__ uint8_t ac_raw[];
  __shared__ __align__(8) uint64_t bars[kAcWarps][kAcStages];
  __shared__ float s_m[kAcWarps][16], s_l[kAcWarps][16];
  __shared__ float c_m[16], c_l[16];
  uint8_t* smem = ac_raw + ((1024u - (smem_u32(ac_raw) & 1023u)) & 1023u);   // 1024-aligned (swizzle atom)
  uint8_t* sQ = smem + kAcWarps * kAcStages * SH::SB;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int cs = a.splits;
  const int seg = blockIdx.x / cs;
  uint32_t crank;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  const int b = seg / a.kv_heads;
  const int hk = seg - b * a.kv_heads;
  const int G = a.q_heads / a.kv_heads;
  const int nr = a.nr;
  int count = a.counts ? a.counts[seg] : a.num_sel;
  if (count > a.num_sel) count = a.num_sel;
  if (count < 0) count = 0;
  const int rb = (int)crank * a.rps;
  const int re = min(count, rb + a.rps);
  const int nblk = re > rb ? (re - rb + kAcBlock - 1) / kAcBlock : 0;
  const int nw = nblk > warp ? (nblk - warp + kAcWarps - 1) / kAcWarps : 0;   // this warp's blocks

  uint8_t* wst = smem + warp * kAcStages * SH::SB;     // this warp's stages
  const uint32_t bar0 = smem_u32(&bars[warp][0]);     // stage s's mbarrier: bar0 + 8 s
  auto issue = [&](int i) {                            // lane 0: block i of this warp into its stage
    const int s = i % kAcStages;
    const int y = rb + (warp + kAcWarps * i) * kAcBlock;
    const uint32_t dk = smem_u32(wst + s * SH::SB), dv = dk + SH::KB;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar0 + 8 * s), "r"(SH::SB) : "memory");
#pragma unroll
    for (int h = 0; h < SH::HALVES; ++h) {
      ac_tma_load(dk + h * SH::HB, &tk, h * 64, y, seg, bar0 + 8 * s);
      ac_tma_load(dv + h * SH::HB, &tv, h * 64, y, seg, bar0 + 8 * s);
    }
  };
  // query rows (zero beyond nr) in 16-byte chunks, requested before the block loads so they do
  // not queue behind them
  constexpr int CPR = D * 2 / 16;
  constexpr int QPT = 16 * CPR / (kAcWarps * 32);      // chunks per thread
  uint4 qv[QPT];
#pragma unroll
  for (int k = 0; k < QPT; ++k) {
    const int x = tid + k * kAcWarps * 32;
    const int r = x / CPR, c = x - r * CPR;
    qv[k] = make_uint4(0, 0, 0, 0);
    if (r < nr) {
      const int gq = r / a.q_len, i = r - gq * a.q_len;
      qv[k] = *reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.q_sb + (int64_t)(hk * G + gq) * a.q_sh +
                                              (int64_t)i * a.q_sq + c * 16);
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kAcStages; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < nw && i < kAcStages; ++i) issue(i);
  }
#pragma unroll
  for (int k = 0; k < QPT; ++k) {
    const int x = tid + k * kAcWarps * 32;
    const int r = x / CPR, c = x - r * CPR;
    *reinterpret_cast<uint4*>(sQ + r * SH::ROWP + c * 16) = qv[k];
  }
  __syncthreads();
  // Q fragments.  Wide (9..16 query rows): Q is the A operand (query rows on M = 16).  Narrow
  // (<= 8 query rows): the block's 16 selected rows go on M and the query rows on N = 8, so no
  // MMA row is padding: S^T = K·Q^T and O^T = V^T·P^T, Q the B operand.
  constexpr int NA = NARROW ? D / 16 : D / 8;          // accumulator tiles of O (or O^T)
  uint32_t qf[KS][NARROW ? 2 : 4];
#pragma unroll
  for (int kk = 0; kk < KS; kk += (NARROW ? 2 : 1)) {
    if constexpr (NARROW) {
      uint32_t t[4];
      ldsm_x4(t, sQ + (lane & 7) * SH::ROWP + (2 * kk + (lane >> 3)) * 16);
      qf[kk][0] = t[0];
      qf[kk][1] = t[1];
      qf[kk + 1][0] = t[2];
      qf[kk + 1][1] = t[3];
    } else {
      const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
      ldsm_x4(qf[kk], sQ + row * SH::ROWP + (2 * kk + (lane >> 4)) * 16);
    }
  }

  const float sl2 = a.scale * 1.4426950408889634f;     // exponent base 2: exp(x) = 2^(x log2 e)
  // running max / normaliser of the thread's two query rows: wide, rows g and g + 8; narrow,
  // query columns 2 tig and 2 tig + 1
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[NA][4];
#pragma unroll
  for (int n = 0; n < NA; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  bool ok = true;
  for (int i = 0; i < nw; ++i) {
    const int s = i % kAcStages;
    uint32_t done = 0;
    if (lane == 0) done = ac_wait(bar0 + 8 * s, (uint32_t)(i / kAcStages) & 1u);
    done = __shfl_sync(0xffffffffu, done, 0);
    if (!done) {                                       // record it, let the other loads land, stop
      if (lane == 0) {
        if (a.status) atomicOr(a.status, MSKV_STATUS_TIMEOUT);
        for (int j = i; j < nw && j < i + kAcStages; ++j)
          ac_wait(bar0 + 8 * (j % kAcStages), (uint32_t)(j / kAcStages) & 1u);
      }
      __syncwarp();
      ok = false;
      break;
    }
    uint8_t* sK = wst + s * SH::SB;
    uint8_t* sV = sK + SH::KB;
    const int y0 = rb + (warp + kAcWarps * i) * kAcBlock;
    const int vrows = min(kAcBlock, re - y0);
    if (vrows < kAcBlock) {                            // rows past the count: zero V
      for (int x = lane; x < (kAcBlock - vrows) * 8 * SH::HALVES; x += 32) {
        const int r = vrows + x / (8 * SH::HALVES), c = x % (8 * SH::HALVES);
        *reinterpret_cast<uint4*>(sV + ac_swz(r, c)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    // scores: sc[e] of the thread's C fragment, scaled to base 2, masked past the block's rows.
    // Wide: C = S (query g / g+8 x block rows 8j + 2 tig + {0,1}), two n-tiles j.  Narrow:
    // C = S^T (block rows g / g+8 x query columns 2 tig + {0,1}).  K-steps accumulate in
    // separate chains and are summed at the end.
    constexpr int NJ = NARROW ? 1 : 2;
    constexpr int CH = NARROW ? 4 : 2;                 // accumulation chains per n-tile
    float sacc[NJ][CH][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int c = 0; c < CH; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[j][c][e] = 0.f;
    if constexpr (NARROW) {
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t ka[4];
        const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
        ldsm_x4(ka, sK + ac_swz(row, 2 * kk + (lane >> 4)));
        mma16816<BF16>(sacc[0][kk % CH], ka, qf[kk][0], qf[kk][1]);
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < KS; kk += 2) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t kb[4];
          ldsm_x4(kb, sK + ac_swz(8 * j + (lane & 7), 2 * kk + (lane >> 3)));
          mma16816<BF16>(sacc[j][0], qf[kk], kb[0], kb[1]);
          mma16816<BF16>(sacc[j][1], qf[kk + 1], kb[2], kb[3]);
        }
      }
    }
    float sc[NJ][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = 0.f;
#pragma unroll
        for (int c = 0; c < CH; ++c) v += sacc[j][c][e];
        const int brow = NARROW ? g + 8 * (e >> 1) : 8 * j + 2 * tig + (e & 1);   // block row of the value
        sc[j][e] = brow < vrows ? v * sl2 : -INFINITY;
      }
    // online softmax.  Query row q(e) of value e: wide, e >> 1 (g or g + 8); narrow, e & 1.
    float bm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = NARROW ? (e & 1) : (e >> 1);
        bm[q] = fmaxf(bm[q], sc[j][e]);
      }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if constexpr (NARROW) {                          // across the 8 groups holding the block rows
        bm[q] = fmaxf(bm[q], __shfl_xor_sync(0xffffffffu, bm[q], 4));
        bm[q] = fmaxf(bm[q], __shfl_xor_sync(0xffffffffu, bm[q], 8));
        bm[q] = fmaxf(bm[q], __shfl_xor_sync(0xffffffffu, bm[q], 16));
      } else {                                         // across the 4 lanes sharing a query row
        bm[q] = fmaxf(bm[q], __shfl_xor_sync(0xffffffffu, bm[q], 1));
        bm[q] = fmaxf(bm[q], __shfl_xor_sync(0xffffffffu, bm[q], 2));
      }
    }
    const float mn0 = fmaxf(m[0], bm[0]), mn1 = fmaxf(m[1], bm[1]);   // finite: the block has a row
    const bool moved = __any_sync(0xffffffffu, mn0 != m[0] || mn1 != m[1]);
    float ps[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = NARROW ? (e & 1) : (e >> 1);
        sc[j][e] = ex2(sc[j][e] - (q ? mn1 : mn0));    // masked: 2^-inf = 0
        ps[q] += sc[j][e];
      }
    if (moved) {                                       // rescale what was summed under the old maxima
      const float c0 = ex2(m[0] - mn0), c1 = ex2(m[1] - mn1);   // 0 while nothing was seen, 1 if unchanged
      l[0] *= c0;
      l[1] *= c1;
#pragma unroll
      for (int n = 0; n < NA; ++n) {
        if constexpr (NARROW) {
          acc[n][0] *= c0;
          acc[n][1] *= c1;
          acc[n][2] *= c0;
          acc[n][3] *= c1;
        } else {
          acc[n][0] *= c0;
          acc[n][1] *= c0;
          acc[n][2] *= c1;
          acc[n][3] *= c1;
        }
      }
      m[0] = mn0;
      m[1] = mn1;
    }
    l[0] += ps[0];
    l[1] += ps[1];
    if constexpr (NARROW) {
      // P^T (block rows x query columns, C layout) -> the B operand of O^T += V^T·P^T by one 8x8
      // transpose per half; V^T comes in as the A operand through ldmatrix.trans
      const uint32_t pb0 = movmatrix_trans(pack2<BF16>(sc[0][0], sc[0][1]));
      const uint32_t pb1 = movmatrix_trans(pack2<BF16>(sc[0][2], sc[0][3]));
#pragma unroll
      for (int mt = 0; mt < NA; ++mt) {
        uint32_t va[4];
        ldsm_x4_t(va, sV + ac_swz((lane & 7) + 8 * (lane >> 4), 2 * mt + ((lane >> 3) & 1)));
        mma16816<BF16>(acc[mt], va, pb0, pb1);
      }
    } else {
      // O += P·V: P as the A fragment of one 16-row k-step, V through ldmatrix.trans
      uint32_t pa[4];
      pa[0] = pack2<BF16>(sc[0][0], sc[0][1]);
      pa[1] = pack2<BF16>(sc[0][2], sc[0][3]);
      pa[2] = pack2<BF16>(sc[1][0], sc[1][1]);
      pa[3] = pack2<BF16>(sc[1][2], sc[1][3]);
#pragma unroll
      for (int n = 0; n < NA; n += 2) {
        uint32_t vb[4];
        ldsm_x4_t(vb, sV + ac_swz((lane & 7) + 8 * ((lane >> 3) & 1), n + (lane >> 4)));
        mma16816<BF16>(acc[n], pa, vb[0], vb[1]);
        mma16816<BF16>(acc[n + 1], pa, vb[2], vb[3]);
      }
    }
    __syncwarp();                                      // every lane has read the stage
    if (lane == 0 && i + kAcStages < nw) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // reads/zeroes before the refill
      issue(i + kAcStages);
    }
  }
  if (!ok) {
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
#pragma unroll
    for (int n = 0; n < NA; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if constexpr (NARROW) {
      l[q] += __shfl_xor_sync(0xffffffffu, l[q], 4);
      l[q] += __shfl_xor_sync(0xffffffffu, l[q], 8);
      l[q] += __shfl_xor_sync(0xffffffffu, l[q], 16);
    } else {
      l[q] += __shfl_xor_sync(0xffffffffu, l[q], 1);
      l[q] += __shfl_xor_sync(0xffffffffu, l[q], 2);
    }
  }
  // the warp's partial -> its first two stages (all its loads have landed): O as [query row][dim]
  float* so = reinterpret_cast<float*>(wst);
  if constexpr (NARROW) {
#pragma unroll
    for (int mt = 0; mt < NA; ++mt) {
      so[(2 * tig) * OS + mt * 16 + g] = acc[mt][0];
      so[(2 * tig + 1) * OS + mt * 16 + g] = acc[mt][1];
      so[(2 * tig) * OS + mt * 16 + g + 8] = acc[mt][2];
      so[(2 * tig + 1) * OS + mt * 16 + g + 8] = acc[mt][3];
    }
    if (g == 0) {
      s_m[warp][2 * tig] = m[0];
      s_m[warp][2 * tig + 1] = m[1];
      s_l[warp][2 * tig] = l[0];
      s_l[warp][2 * tig + 1] = l[1];
    }
  } else {
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const int col = n * 8 + 2 * tig;
      *reinterpret_cast<float2*>(so + g * OS + col) = make_float2(acc[n][0], acc[n][1]);
      *reinterpret_cast<float2*>(so + (g + 8) * OS + col) = make_float2(acc[n][2], acc[n][3]);
    }
    if (tig == 0) {
      s_m[warp][g] = m[0];
      s_m[warp][g + 8] = m[1];
      s_l[warp][g] = l[0];
      s_l[warp][g + 8] = l[1];
    }
  }
  __syncthreads();
  // four warps -> the CTA's partial (warp 0's third stage, which no warp uses any more): one pass,
  // four output dims per thread, every input requested before the first is used
  constexpr int D4 = D / 4;
  float* co = reinterpret_cast<float*>(smem + 2 * SH::SB);
  for (int x = tid; x < nr * D4; x += kAcWarps * 32) {
    const int r = x / D4, d = (x - r * D4) * 4;
    float mw[kAcWarps], lw[kAcWarps];
    float4 ow[kAcWarps];
#pragma unroll
    for (int w = 0; w < kAcWarps; ++w) {
      mw[w] = s_m[w][r];
      lw[w] = s_l[w][r];
      ow[w] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(smem + w * kAcStages * SH::SB) + r * OS + d);
    }
    float M = mw[0];
#pragma unroll
    for (int w = 1; w < kAcWarps; ++w) M = fmaxf(M, mw[w]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kAcWarps; ++w) {
      const float f = mw[w] == -INFINITY ? 0.f : exp2f(mw[w] - M);
      L += lw[w] * f;
      o.x += ow[w].x * f;
      o.y += ow[w].y * f;
      o.z += ow[w].z * f;
      o.w += ow[w].w * f;
    }
    *reinterpret_cast<float4*>(co + r * D + d) = o;
    if (d == 0) {
      c_m[r] = M;
      c_l[r] = L;
    }
  }
  if (cs > 1) cluster_sync_all();
  else __syncthreads();
  // the cluster's CTAs -> the output.  Query row r is finished by CTA r mod cs, four dims per
  // thread; the D/4 lanes that share a row fetch the cs peers' maxima and normalisers once
  // (lane q of the group from peer q) and pass them on with shuffles, and every peer's four dims
  // are requested before the first is used.
  static_assert(D4 >= kAcMaxCluster && 32 % D4 == 0, "a row's lanes must cover the cluster");
  const uint32_t co_a = smem_u32(co), cm_a = smem_u32(c_m), cl_a = smem_u32(c_l);
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int my_rows = nr > (int)crank ? (nr - (int)crank + cs - 1) / cs : 0;
  const int gbase = lane & ~(D4 - 1), li = lane & (D4 - 1);     // this lane's row group in the warp
  for (int y0 = warp * 32; y0 < my_rows * D4; y0 += kAcWarps * 32) {   // warp-uniform trip count
    const int y = y0 + lane;
    const bool live = y < my_rows * D4;
    const int r = live ? (int)crank + cs * (y / D4) : (int)crank;
    const int d = (y % D4) * 4;
    float mine_m = -INFINITY, mine_l = 0.f;
    if (li < cs) {
      mine_m = cs == 1 ? c_m[r] : ld_cluster_f32(cm_a + 4 * r, li);
      mine_l = cs == 1 ? c_l[r] : ld_cluster_f32(cl_a + 4 * r, li);
    }
    float4 oq[kAcMaxCluster];
#pragma unroll
    for (int q = 0; q < kAcMaxCluster; ++q)
      if (q < cs) oq[q] = cs == 1 ? *reinterpret_cast<const float4*>(co + r * D + d) : ld_cluster_f32x4(co_a + 4 * (r * D + d), q);
    float mq[kAcMaxCluster], lq[kAcMaxCluster];
#pragma unroll
    for (int q = 0; q < kAcMaxCluster; ++q) {
      mq[q] = __shfl_sync(0xffffffffu, mine_m, gbase + q);
      lq[q] = __shfl_sync(0xffffffffu, mine_l, gbase + q);
    }
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kAcMaxCluster; ++q)
      if (q < cs) M = fmaxf(M, mq[q]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < kAcMaxCluster; ++q) {
      if (q < cs && mq[q] != -INFINITY) {
        const float f = exp2f(mq[q] - M);
        L += lq[q] * f;
        o.x += oq[q].x * f;
        o.y += oq[q].y * f;
        o.z += oq[q].z * f;
        o.w += oq[q].w * f;
      }
    }
    if (live) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      const int gq = r / a.q_len, i = r - gq * a.q_len;
      T* op = reinterpret_cast<T*>(a.out + (int64_t)b * a.o_sb + (int64_t)(hk * G + gq) * a.o_sh + (int64_t)i * a.o_sq) + d;
      op[0] = from_f<T>(o.x * inv);
      op[1] = from_f<T>(o.y * inv);
      op[2] = from_f<T>(o.z * inv);
      op[3] = from_f<T>(o.w * inv);
    }
  }
  if (cs > 1) cluster_sync_all();                      // no CTA leaves while a peer reads its partial
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

// ---- streaming cluster path: tensor maps and the split -------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library links only the
// runtime); nullptr when the driver does not offer it.
static EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
    cudaGetLastError();
  });
  return fn;
}

// K or V rows as a 3-D tensor [segment][row][dim] of 16-bit elements with 16-row x 64-element
// boxes and the 128-byte swizzle; rows past the width read as zeros.
static bool encode_rows_map(CUtensorMap* m, const void* base, const mskv_attn_desc* d) {
  const int64_t segs = (int64_t)d->batch * d->kv_heads;
  const int64_t seg_stride = segs > 1 ? d->kv_stride_seg : (int64_t)d->num_selected * d->kv_stride_s;
  const cuuint64_t dims[3] = {(cuuint64_t)d->head_dim, (cuuint64_t)d->num_selected, (cuuint64_t)segs};
  const cuuint64_t strides[2] = {(cuuint64_t)d->kv_stride_s, (cuuint64_t)seg_stride};
  const cuuint32_t box[3] = {64, (cuuint32_t)kAcBlock, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return tensor_map_encoder()(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct ClusterPlan {
  bool use;
  int cs;     // CTAs per segment (the cluster)
  int rps;    // selected rows per CTA, a multiple of the 16-row block
  CUtensorMap tk, tv;
};

// The split depends only on the selection width: cs = ceil(width / 256) CTAs (at most 8), each
// with an equal multiple of 16 rows.  Selections wider than 8 x 4096 rows, empty ones, and rows
// the TMA unit cannot address (strides not multiples of 16 bytes, checked by fast_path, or a
// layout the tensor-map encoder refuses) take the split path.
static void cluster_plan(const mskv_attn_desc* d, ClusterPlan* p) {
  p->use = false;
  if (!fast_path(d) || d->num_selected <= 0 || d->num_selected > kAcMaxWidth || d->batch <= 0) return;
  if (d->kv_stride_s < d->head_dim * 2 || (d->batch * (int64_t)d->kv_heads > 1 && d->kv_stride_seg <= 0)) return;
  if (!tensor_map_encoder() || !encode_rows_map(&p->tk, d->k, d) || !encode_rows_map(&p->tv, d->v, d)) return;
  const int w = d->num_selected;
  p->cs = std::min(kAcMaxCluster, std::max(1, (w + kAcRowsPerCta - 1) / kAcRowsPerCta));
  const int blocks = (w + kAcBlock - 1) / kAcBlock;
  p->rps = ((blocks + p->cs - 1) / p->cs) * kAcBlock;
  p->use = true;
}

template <bool BF16, int D, bool NARROW>
static int launch_cluster(const AttnDev& a, const mskv_attn_desc* d, const ClusterPlan& p, cudaStream_t st) {
  int rc;
  const void* kern = (const void*)attn_cluster_kernel<BF16, D, NARROW>;
  rc = ensure_smem_limit(kern, AcShape<D>::SMEM, "mskv_sparse_attention");
  if (rc) return rc;
  const int64_t blocks = (int64_t)d->batch * d->kv_heads * p.cs;
  if (blocks > 0x7fffffffLL) return fail(MSKV_ERR_RANGE, "mskv_sparse_attention: grid too large");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kAcWarps * 32);
  cfg.dynamicSmemBytes = AcShape<D>::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.cs > 1 ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_cluster_kernel<BF16, D, NARROW>, a, p.tk, p.tv);
  if (e != cudaSuccess) return cuda_status(e, "mskv_sparse_attention cluster launch");
  return after_launch("mskv_sparse_attention");
}

}  // namespace mskv

using namespace mskv;

extern "C" uint64_t mskv_attention_workspace_bytes(const mskv_attn_desc* d) {
  if (!d || d->kv_heads <= 0 || d->q_heads <= 0 || d->q_len <= 0 || d->batch < 0) return 0;
  if (!fast_path(d)) return 0;
  ClusterPlan cp;
  cluster_plan(d, &cp);
  if (cp.use) return 0;
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
  ClusterPlan cp;
  cluster_plan(d, &cp);
  if (cp.use) {
    a.splits = cp.cs;
    a.rps = cp.rps;
    const bool bf = d->dtype == MSKV_DT_BF16;
    if (a.nr <= 8) {
      if (d->head_dim == 128) return bf ? launch_cluster<true, 128, true>(a, d, cp, st) : launch_cluster<false, 128, true>(a, d, cp, st);
      return bf ? launch_cluster<true, 64, true>(a, d, cp, st) : launch_cluster<false, 64, true>(a, d, cp, st);
    }
    if (d->head_dim == 128) return bf ? launch_cluster<true, 128, false>(a, d, cp, st) : launch_cluster<false, 128, false>(a, d, cp, st);
    return bf ? launch_cluster<true, 64, false>(a, d, cp, st) : launch_cluster<false, 64, false>(a, d, cp, st);
  }
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
