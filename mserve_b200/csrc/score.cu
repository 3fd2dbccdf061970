// Importance scoring of every cached token against the decode query (mskv_score).
//
// The reference computes torch.matmul(q, Kᵀ) over repeat_kv'd heads and averages over all
// query heads (qwen-eljrte/Qwen_Transformer/attention.py:558-565).  Here the GQA group is
// folded first: sum_g q_g·k = (sum_g q_g)·k, so every K element is read once from HBM and
// costs one FMA.  The kernel is a memory-bound GEMV (tensor cores are deliberately unused):
//
//  * a group of GL lanes (GL = 16 for bf16 D=128) owns GL consecutive rows per iteration;
//    lane l loads the l-th 16-byte chunk of each of those rows (GL independent 16-byte loads
//    in flight per lane, 256 contiguous bytes per row per instruction), converts to fp32 and
//    accumulates one partial dot product per row;
//  * a butterfly reduce-scatter over the GL lanes (GL-1 shuffles for GL rows instead of
//    GL*log2(GL)) leaves lane l holding the full fp32 score of row l, so a warp writes its
//    32 scores as one coalesced 128-byte store;
//  * warps own contiguous runs of 32-row slices, so the GQA-summed query is rebuilt only when
//    a warp crosses into a new (b, KV head) segment.
#include "common.cuh"
#include "tma.cuh"

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
};

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
    if (group_ok && t < len) a.scores[seg * a.scores_stride + t] = score;
  }
}

// Generic path: any head_dim, element-wise loads, one warp per row.
template <typename T, int METHOD>
__global__ void __launch_bounds__(256) score_generic_kernel(const ScoreDev a) {
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
    if (lane == 0) a.scores[seg * a.scores_stride + t] = METHOD == 1 ? sqrtf(acc) : acc;
  }
}

// ---------------------------------------------------------------------------------------
// Bulk-copy (TMA) pipeline: the main path for 16-bit keys with contiguous rows.
//
// A persistent CTA of 128 threads owns a contiguous, balanced range of 128-token tiles
// (tiles of one (b, KV head) segment are consecutive).  Warp 0 streams tiles into a ring of
// STAGES shared-memory buffers with cp.async.bulk (paged keys: one 4 KB copy per page and
// head, issued by one lane per page; strided keys: one copy per tile), each stage guarded by
// an mbarrier with transaction counting.  All four warps score the resident tile: a 16-lane
// group reads 16 rows as 16-byte chunks (256 contiguous bytes per row, conflict-free), and
// the same butterfly reduce-scatter as above leaves each lane with one row's score.  Two
// CTAs per SM keep up to 6 x 32 KB of key bytes in flight.
template <int D>
struct TmaCfg {
  static constexpr int ROWB = D * 2;
  static constexpr int TILE = 128;
  static constexpr int STAGES = D == 64 ? 4 : 3;
  static constexpr int STAGE_BYTES = TILE * ROWB;
  static constexpr int SMEM = STAGES * STAGE_BYTES;
};

struct TmaTile {
  int64_t seg, t0;
  int b, h;
  int nv;  // valid rows in the tile
};

__device__ __forceinline__ TmaTile tma_tile(const ScoreDev& a, int64_t tile, int64_t tiles_per_seg, int tile_rows) {
  TmaTile t;
  t.seg = tile / tiles_per_seg;
  t.t0 = (tile - t.seg * tiles_per_seg) * tile_rows;
  t.b = (int)(t.seg / a.kv_heads);
  t.h = (int)(t.seg - (int64_t)t.b * a.kv_heads);
  const int64_t L = rows_len(a.k, t.b);
  const int64_t nv = L - t.t0;
  t.nv = nv <= 0 ? 0 : (nv > tile_rows ? tile_rows : (int)nv);
  return t;
}

template <typename T, int D, int METHOD, bool PAGED>
__global__ void __launch_bounds__(128) score_tma_kernel(const ScoreDev a, uint32_t* status) {
  using Cfg = TmaCfg<D>;
  constexpr int EPV = 8;
  constexpr int LPR = D / EPV;
  constexpr int GL = LPR < 16 ? LPR : 16;
  constexpr int VPL = LPR / GL;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[Cfg::STAGES];
  __shared__ uint32_t s_pages_ok[Cfg::STAGES];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane & (GL - 1), grp = lane / GL;
  const int64_t tiles_per_seg = (a.max_tokens + Cfg::TILE - 1) / Cfg::TILE;
  const int64_t total = (int64_t)a.batch * a.kv_heads * tiles_per_seg;
  const int64_t per = total / gridDim.x, rem = total % gridDim.x;
  const int64_t t_begin = (int64_t)blockIdx.x * per + min((int64_t)blockIdx.x, rem);
  const int64_t t_count = per + ((int64_t)blockIdx.x < rem ? 1 : 0);

  if (tid == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  // Warp 0: start the bulk copies of relative tile i into stage i % STAGES.
  auto issue = [&](int64_t i) {
    const TmaTile tt = tma_tile(a, t_begin + i, tiles_per_seg, Cfg::TILE);
    const int stage = (int)(i % Cfg::STAGES);
    uint8_t* dst = smem + stage * Cfg::STAGE_BYTES;
    uint64_t* bar = &full[stage];
    fence_proxy_async_smem();
    if constexpr (PAGED) {
      const int ps = a.k.page_size;
      const int npages = (tt.nv + ps - 1) / ps;
      uint32_t bytes = 0;
      const char* src = nullptr;
      if (lane < npages) {
        const int64_t pidx = tt.t0 / ps + lane;
        const int32_t page = a.k.page_table[(int64_t)tt.b * a.k.pt_stride + pidx];
        const int rows = min(ps, tt.nv - lane * ps);
        if (page >= 0 && page < a.k.num_pages) {
          bytes = (uint32_t)(rows * Cfg::ROWB);
          src = a.k.base_k + (int64_t)page * a.k.sp + (int64_t)tt.h * a.k.sh;
        } else if (status) {
          atomicOr(status, MSKV_STATUS_BAD_PAGE);
        }
      }
      const uint32_t ok_mask = __ballot_sync(0xffffffffu, bytes > 0);
      uint32_t sum = bytes;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        s_pages_ok[stage] = ok_mask;
        mbar_arrive_expect_tx(bar, sum);
      }
      __syncwarp();
      if (bytes) bulk_load(dst + (int64_t)lane * ps * Cfg::ROWB, src, bytes, bar);
    } else {
      if (lane == 0) {
        const uint32_t bytes = (uint32_t)(tt.nv * Cfg::ROWB);
        s_pages_ok[stage] = 0xffffffffu;
        mbar_arrive_expect_tx(bar, bytes);
        if (bytes)
          bulk_load(dst, a.k.base_k + (int64_t)tt.b * a.k.sb + (int64_t)tt.h * a.k.sh + tt.t0 * a.k.st, bytes, bar);
      }
    }
  };

  if (warp == 0) {
    const int64_t pre = t_count < Cfg::STAGES ? t_count : Cfg::STAGES;
    for (int64_t i = 0; i < pre; ++i) issue(i);
  }

  float qs[VPL][EPV];
  int64_t cur_seg = -1;
  int64_t waited = 0;
  bool timed_out = false;
  for (int64_t i = 0; i < t_count; ++i) {
    const int stage = (int)(i % Cfg::STAGES);
    const bool ok = mbar_wait(&full[stage], (uint32_t)((i / Cfg::STAGES) & 1), kWaitTimeoutNs);
    if (__syncthreads_or(!ok)) {
      timed_out = true;
      break;
    }
    waited = i + 1;
    const TmaTile tt = tma_tile(a, t_begin + i, tiles_per_seg, Cfg::TILE);
    if (tt.seg != cur_seg) {
      cur_seg = tt.seg;
      if constexpr (METHOD == 0) {
        const int G = a.q_heads / a.kv_heads;
#pragma unroll
        for (int v = 0; v < VPL; ++v)
#pragma unroll
          for (int e = 0; e < EPV; ++e) qs[v][e] = 0.f;
        for (int g = 0; g < G; ++g) {
          const char* qrow = a.q + (int64_t)tt.b * a.q_sb + (int64_t)(tt.h * G + g) * a.q_sh;
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
    const uint8_t* tile_smem = smem + stage * Cfg::STAGE_BYTES;
    const uint32_t pages_ok = s_pages_ok[stage];
#pragma unroll
    for (int half = 0; half < Cfg::TILE / 128; ++half) {
      const int rbase = half * 128 + warp * 32 + grp * GL;
      float part[GL];
#pragma unroll
      for (int j = 0; j < GL; ++j) {
        const int row = rbase + j;
        float acc = 0.f;
        if (row < tt.nv) {
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            const uint4 raw = *reinterpret_cast<const uint4*>(tile_smem + row * Cfg::ROWB + (gl + v * GL) * 16);
            float f[EPV];
            Cvt<T>::to_f32(raw, f);
#pragma unroll
            for (int e = 0; e < EPV; ++e) {
              if constexpr (METHOD == 0) acc = fmaf(qs[v][e], f[e], acc);
              else acc = fmaf(f[e], f[e], acc);
            }
          }
        }
        part[j] = acc;
      }
      float sc = reduce_scatter<GL>(part, gl);
      if constexpr (METHOD == 1) sc = sqrtf(sc);
      const int row = half * 128 + warp * 32 + lane;
      if (row < tt.nv) {
        bool valid = true;
        if constexpr (PAGED) valid = (pages_ok >> (row / a.k.page_size)) & 1u;
        a.scores[tt.seg * a.scores_stride + tt.t0 + row] = valid ? sc : -INFINITY;
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (warp == 0 && i + Cfg::STAGES < t_count) issue(i + Cfg::STAGES);
  }
  if (timed_out) {
    if (tid == 0 && status) atomicOr(status, MSKV_STATUS_TIMEOUT);
    // Let copies still in flight land before the CTA's shared memory is released.
    const int64_t issued = t_count < waited + Cfg::STAGES ? t_count : waited + Cfg::STAGES;
    for (int64_t i = waited; i < issued; ++i)
      mbar_wait(&full[i % Cfg::STAGES], (uint32_t)((i / Cfg::STAGES) & 1), kDrainTimeoutNs);
  }
}

template <typename T, int D, int METHOD, bool PAGED>
static int launch_tma(ScoreDev& a, uint32_t* status, cudaStream_t st) {
  using Cfg = TmaCfg<D>;
  auto kern = score_tma_kernel<T, D, METHOD, PAGED>;
  static bool attr_set = false;  // benign race: every thread sets the same value
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set = true;
  }
  int occ = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 128, Cfg::SMEM);
  if (occ < 1) occ = 1;
  const int64_t tiles = (int64_t)a.batch * a.kv_heads * ((a.max_tokens + Cfg::TILE - 1) / Cfg::TILE);
  int64_t grid = (int64_t)num_sms() * occ;
  if (grid > tiles) grid = tiles;
  if (grid < 1) grid = 1;
  kern<<<(unsigned)grid, 128, Cfg::SMEM, st>>>(a, status);
  return after_launch("mskv_score");
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
static int dispatch_d(ScoreDev& a, bool paged, bool fast, bool tma, uint32_t* status, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    if (tma) {
#define MSKV_TMA_CASE(DD)                                                              \
  if (a.head_dim == DD) return paged ? launch_tma<T, DD, METHOD, true>(a, status, st)  \
                                     : launch_tma<T, DD, METHOD, false>(a, status, st);
      MSKV_TMA_CASE(64)
      MSKV_TMA_CASE(128)
      MSKV_TMA_CASE(256)
#undef MSKV_TMA_CASE
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
static int dispatch_method(ScoreDev& a, bool paged, bool fast, bool tma, uint32_t* status, cudaStream_t st) {
  return a.method == 0 ? dispatch_d<T, 0>(a, paged, fast, tma, status, st)
                       : dispatch_d<T, 1>(a, paged, fast, tma, status, st);
}

}  // namespace mskv

using namespace mskv;

extern "C" int mskv_score(const mskv_score_desc* d, void* stream) {
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
  const bool paged = d->k.page_table != nullptr;
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
  // The bulk-copy pipeline also needs contiguous rows (a tile or page is one copy) and, when
  // paged, pages of 4..128 tokens that tile the 128-token key tiles exactly.
  bool tma = fast && es == 2 && d->k.stride_t == (int64_t)d->head_dim * es &&
             (d->head_dim == 64 || d->head_dim == 128 || d->head_dim == 256);
  if (paged) tma = tma && d->k.page_size >= 4 && d->k.page_size <= 128 && (128 % d->k.page_size) == 0;
  cudaStream_t st = as_stream(stream);
  switch (d->dtype) {
    case MSKV_DT_F32: return dispatch_method<float>(a, paged, fast, false, d->status, st);
    case MSKV_DT_F16: return dispatch_method<__half>(a, paged, fast, tma, d->status, st);
    default: return dispatch_method<__nv_bfloat16>(a, paged, fast, tma, d->status, st);
  }
}
