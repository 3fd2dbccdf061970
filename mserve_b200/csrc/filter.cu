// Image-token filter of a prefill attention map (mskv_image_filter).
//
// Replaces dual_attention_filter (qwen-eljrte/Qwen_Transformer/dual_attention_filter.py:6-103):
// from the attention probabilities of batch 0, the block of text rows x image columns
// [H, text, img] is averaged over the heads; per image token the column sum over the text rows
// (the "global" score) and the column maximum (the "individual" score) decide whether it is
// dropped:  drop = sum < total * global_thr  and  max < individual_thr,  total = the sum of
// all column sums.  The kept image tokens are returned in ascending order.
//
// Stage precision.  The reference computes each stage as a torch tensor of the block's dtype
// (fp16 after its optional .half()): the head mean, the column sums and maxima, the total and
// total * global_thr are each rounded to that dtype, with fp32 accumulation inside each
// reduction.  The kernels do the same: fp32 sums, the stage results rounded to the stage
// dtype (fp32, fp16 or bf16).  individual_thr is rounded to the stage dtype too: torch casts a
// Python scalar to the tensor's dtype before `text_max < individual_thr`, so for a 16-bit block
// a threshold that rounds down (bf16(0.001) = 0.00099945...) keeps a column whose maximum
// equals the rounded value.
//
// Summation order, fixed (so the result does not depend on the launch shape):
//   head mean   hm[i,j] = stage((sum over heads in order) / H)
//   column sum  the text rows in blocks of 32; each block summed in row order, the block sums
//               added in block order; then stage()
//   total       the columns in tiles of 32: each tile summed in column order, the tile sums
//               added in tile order; then stage()
//
// One kernel.  Each thread takes one (text row, image column), so that the whole block is
// requested at once (a prefill map's rows are rarely 16-byte aligned, which rules out vector
// and tensor-map loads; a warp's loads of one (head, row) are 32 consecutive keys, one 128-byte
// line), and issues the loads of 16 heads before adding them in order.  CTA = 32 columns (one
// tile) x up to 32 text rows (one row block); the rows' head means meet in shared memory and
// warp 0 sums them per column.  Completion runs on arrival counters that the host zeroes
// before the launch:
//  * the last CTA of a tile to finish combines the tile's row blocks per column (the only CTA
//    when the text fits one block), writes the column sums and maxima and the tile's share;
//  * the last tile to finish sums the shares, applies the thresholds and compacts the kept
//    columns in order through ballots and a warp scan, with the kept-decision inputs of its
//    first rounds loaded before the total is known.
#include "common.cuh"

namespace mskv {

struct FilterDev {
  const char* attn;
  int64_t sh, sq, sk;            // element strides of head, query row, key column (batch 0)
  int32_t heads, txt_beg, text, img_beg, img, nblocks, ntiles;
  float global_thr, individual_thr;
  uint32_t* arrivals;            // [ntiles] per tile, then [1] tiles done: zero before the launch
  float* part_sum;               // [nblocks][img]
  float* part_max;               // [nblocks][img]
  float* col_sum;
  float* col_max;
  float* tile_sums;
  int64_t* out_idx;
  int32_t* out_count;
};

constexpr int kRowBlock = 32;                // text rows per block (summed in order)
constexpr int kHeadBatch = 16;               // heads loaded before they are added
constexpr int kSmemTiles = 2048;             // tile shares kept in shared memory (65536 columns)
constexpr int kPrefetchRounds = 2;           // compaction rounds whose inputs load early

enum Stage { kStageF32 = 0, kStageF16 = 1, kStageBF16 = 2 };

template <int S> __device__ __forceinline__ float stage(float x) {
  if constexpr (S == kStageF16) return __half2float(__float2half_rn(x));
  else if constexpr (S == kStageBF16) return __bfloat162float(__float2bfloat16_rn(x));
  else return x;
}

template <typename T> __device__ __forceinline__ float as_f32(T x);
template <> __device__ __forceinline__ float as_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float as_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float as_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// Warp 0 (lane = column of the tile): the finished column's sum s (already staged) and max m;
// writes them and the tile's share, the 32 sums added in column order.
__device__ __forceinline__ void finish_column(const FilterDev& a, int j, float s, float m) {
  if (j < a.img) {
    a.col_sum[j] = s;
    a.col_max[j] = m;
  }
  const float v = j < a.img ? s : 0.f;
  float t = 0.f;
#pragma unroll
  for (int c = 0; c < 32; ++c) t += __shfl_sync(0xffffffffu, v, c);
  if ((threadIdx.x & 31) == 0) a.tile_sums[j >> 5] = t;
}

// One compaction round over columns [j0, j0 + blockDim.x): thread tid decides column j0 + tid.
__device__ __forceinline__ void compact_round(const FilterDev& a, int j, bool keep, uint32_t& base,
                                              uint32_t* s_wcnt, uint32_t* s_wpre, uint32_t* s_round) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const uint32_t m = __ballot_sync(0xffffffffu, keep);
  if (lane == 0) s_wcnt[warp] = __popc(m);
  __syncthreads();
  if (warp == 0) {
    const uint32_t c = lane < nw ? s_wcnt[lane] : 0u;
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    s_wpre[lane] = incl - c;
    if (lane == 31) *s_round = incl;
  }
  __syncthreads();
  uint32_t lt;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
  if (keep) a.out_idx[base + s_wpre[warp] + __popc(m & lt)] = j;
  base += *s_round;
  __syncthreads();   // the round's shared words are rewritten next round
}

// The last tile: total, thresholds, ordered compaction.  The column sums and maxima are read
// through L2 (__ldcg), where the other CTAs' stores are visible after the counters' fences.
template <int S>
__device__ void filter_finish(const FilterDev& a) {
  __shared__ float s_thr;
  __shared__ uint32_t s_wcnt[32], s_wpre[32], s_round;
  __shared__ float s_tiles[kSmemTiles];
  const int nt = blockDim.x, tid = threadIdx.x;
  const bool tiles_in_smem = a.ntiles <= kSmemTiles;
  if (tiles_in_smem)
    for (int c = tid; c < a.ntiles; c += nt) s_tiles[c] = __ldcg(a.tile_sums + c);
  float pcs[kPrefetchRounds], pcm[kPrefetchRounds];
#pragma unroll
  for (int r = 0; r < kPrefetchRounds; ++r) {
    const int j = r * nt + tid;
    pcs[r] = j < a.img ? __ldcg(a.col_sum + j) : 0.f;
    pcm[r] = j < a.img ? __ldcg(a.col_max + j) : 0.f;
  }
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    if (tiles_in_smem) {
#pragma unroll 8
      for (int c = 0; c < a.ntiles; ++c) t += s_tiles[c];
    } else {
#pragma unroll 8
      for (int c = 0; c < a.ntiles; ++c) t += __ldcg(a.tile_sums + c);
    }
    s_thr = stage<S>(stage<S>(t) * a.global_thr);
  }
  __syncthreads();
  const float thr = s_thr;
  const float ithr = stage<S>(a.individual_thr);
  uint32_t base = 0;
#pragma unroll
  for (int r = 0; r < kPrefetchRounds; ++r) {
    if (r * nt >= a.img) break;
    const int j = r * nt + tid;
    const bool keep = j < a.img && !(pcs[r] < thr && pcm[r] < ithr);
    compact_round(a, j, keep, base, s_wcnt, s_wpre, &s_round);
  }
  for (int j0 = kPrefetchRounds * nt; j0 < a.img; j0 += nt) {
    const int j = j0 + tid;
    const bool keep = j < a.img && !(__ldcg(a.col_sum + j) < thr && __ldcg(a.col_max + j) < ithr);
    compact_round(a, j, keep, base, s_wcnt, s_wpre, &s_round);
  }
  if (tid == 0) *a.out_count = (int32_t)base;
}

// S is the stage dtype; for fp32 input with the fp16 rounding mode the elements are rounded to
// fp16 as they load (stage<S> of an fp32 value), which equals the reference's block.half().
// blockDim = 32 x min(32, text): lane = image column, warp = text row of the block.
template <typename T, int S>
__global__ void __launch_bounds__(32 * kRowBlock, 2) filter_kernel(const FilterDev a) {
  __shared__ float s_hm[kRowBlock][33];
  __shared__ bool s_flag;
  const int lane = threadIdx.x & 31, r = threadIdx.x >> 5;
  const int tile = blockIdx.x;
  const int j = tile * 32 + lane;
  const int i = blockIdx.y * kRowBlock + r;
  float hm = 0.f;
  if (j < a.img && i < a.text) {
    const T* p = reinterpret_cast<const T*>(a.attn) + (int64_t)(a.txt_beg + i) * a.sq +
                 (int64_t)(a.img_beg + j) * a.sk;
    const int64_t sh = a.sh;
    float hs = 0.f;
    int h = 0;
    for (; h + kHeadBatch <= a.heads; h += kHeadBatch) {
      T v[kHeadBatch];
#pragma unroll
      for (int u = 0; u < kHeadBatch; ++u) v[u] = __ldg(p + u * sh);
      p += kHeadBatch * sh;
#pragma unroll
      for (int u = 0; u < kHeadBatch; ++u) hs += stage<S>(as_f32<T>(v[u]));
    }
    const int rem = a.heads - h;
    if (rem > 0) {
      T v[kHeadBatch];
#pragma unroll
      for (int u = 0; u < kHeadBatch; ++u)
        if (u < rem) v[u] = __ldg(p + u * sh);
#pragma unroll
      for (int u = 0; u < kHeadBatch; ++u)
        if (u < rem) hs += stage<S>(as_f32<T>(v[u]));
    }
    hm = stage<S>(hs / (float)a.heads);
  }
  s_hm[r][lane] = hm;
  __syncthreads();
  float s = 0.f, m = -INFINITY;   // warp 0: this row block's sum and max of column j
  if (r == 0) {
    const int rows = min(kRowBlock, a.text - (int)blockIdx.y * kRowBlock);
    for (int q = 0; q < rows; ++q) {
      const float x = s_hm[q][lane];
      s += x;
      m = fmaxf(m, x);
    }
  }
  if (a.nblocks == 1) {
    if (r == 0) finish_column(a, j, stage<S>(s), m);
  } else {
    if (r == 0 && j < a.img) {
      a.part_sum[(int64_t)blockIdx.y * a.img + j] = s;
      a.part_max[(int64_t)blockIdx.y * a.img + j] = m;
    }
    // warp 0's partials are published before the tile's counter moves
    if (r == 0) __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_flag = atomicAdd(a.arrivals + tile, 1u) == (uint32_t)a.nblocks - 1;
    __syncthreads();
    if (!s_flag) return;
    if (r == 0) {                 // the tile's row blocks, in block order
      __threadfence();
      float cs = 0.f, cm = -INFINITY;
      if (j < a.img) {
        const float* ps = a.part_sum + j;
        const float* pm = a.part_max + j;
        int b = 0;
        for (; b + 4 <= a.nblocks; b += 4) {
          float vs[4], vm[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            vs[u] = __ldcg(ps + (int64_t)(b + u) * a.img);
            vm[u] = __ldcg(pm + (int64_t)(b + u) * a.img);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            cs += vs[u];
            cm = fmaxf(cm, vm[u]);
          }
        }
        for (; b < a.nblocks; ++b) {
          cs += __ldcg(ps + (int64_t)b * a.img);
          cm = fmaxf(cm, __ldcg(pm + (int64_t)b * a.img));
        }
      }
      finish_column(a, j, stage<S>(cs), cm);
    }
  }
  // the tile is done: warp 0's columns and share are published before the tiles' counter moves
  if (r == 0) __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_flag = atomicAdd(a.arrivals + a.ntiles, 1u) == (uint32_t)a.ntiles - 1;
  __syncthreads();
  if (!s_flag) return;
  __threadfence();              // acquire side: the other tiles' stores are read after this
  filter_finish<S>(a);
}

template <typename T, int S>
static int launch_filter(const FilterDev& a, cudaStream_t st) {
  if (a.img == 0) {            // no image tokens: none kept
    const cudaError_t e = cudaMemsetAsync(a.out_count, 0, sizeof(int32_t), st);
    return e == cudaSuccess ? MSKV_OK : cuda_status(e, "mskv_image_filter memset");
  }
  const cudaError_t e = cudaMemsetAsync(a.arrivals, 0, sizeof(uint32_t) * (a.ntiles + 1), st);
  if (e != cudaSuccess) return cuda_status(e, "mskv_image_filter memset");
  const dim3 grid(a.ntiles, a.nblocks), block(32 * min(kRowBlock, a.text));
  filter_kernel<T, S><<<grid, block, 0, st>>>(a);
  return after_launch("mskv_image_filter");
}

}  // namespace mskv

using namespace mskv;

extern "C" uint64_t mskv_image_filter_workspace_bytes(int32_t img_seq, int32_t text_seq) {
  if (img_seq < 0 || text_seq <= 0) return 0;
  const uint64_t ntiles = ((uint64_t)img_seq + 31) / 32;
  const uint64_t nblocks = ((uint64_t)text_seq + kRowBlock - 1) / kRowBlock;
  const uint64_t counters = (ntiles + 1 + 3) / 4 * 4;     // 16-byte multiple
  return (counters + (2ull * nblocks + 2ull) * (uint64_t)img_seq + ntiles) * sizeof(float);
}

extern "C" int mskv_image_filter(const mskv_filter_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_image_filter: NULL descriptor");
  if (d->heads <= 0 || d->text_seq <= 0 || d->img_seq < 0 || d->img_start < 0 || d->text_start < 0)
    return fail(MSKV_ERR_ARG, "mskv_image_filter: bad sizes (heads and text_seq must be positive)");
  if (d->text_seq > 65535 * kRowBlock) return fail(MSKV_ERR_ARG, "mskv_image_filter: text_seq above %d", 65535 * kRowBlock);
  if (!d->attn || !d->out_idx || !d->out_count) return fail(MSKV_ERR_ARG, "mskv_image_filter: NULL pointer");
  if (!d->workspace || d->workspace_bytes < mskv_image_filter_workspace_bytes(d->img_seq, d->text_seq))
    return fail(MSKV_ERR_ARG, "mskv_image_filter: workspace needs %llu bytes",
                (unsigned long long)mskv_image_filter_workspace_bytes(d->img_seq, d->text_seq));
  if (((uintptr_t)d->workspace & 3) != 0) return fail(MSKV_ERR_ARG, "mskv_image_filter: workspace must be 4-byte aligned");
  if (d->round_f16 && d->dtype != MSKV_DT_F32)
    return fail(MSKV_ERR_ARG, "mskv_image_filter: round_f16 applies to f32 probabilities only");
  FilterDev a{};
  a.attn = static_cast<const char*>(d->attn);
  a.sh = d->stride_h; a.sq = d->stride_q; a.sk = d->stride_k;
  a.heads = d->heads; a.text = d->text_seq; a.img = d->img_seq;
  a.img_beg = d->img_start; a.txt_beg = d->text_start;
  a.global_thr = d->global_thr; a.individual_thr = d->individual_thr;
  a.nblocks = (d->text_seq + kRowBlock - 1) / kRowBlock;
  a.ntiles = (d->img_seq + 31) / 32;
  a.arrivals = static_cast<uint32_t*>(d->workspace);
  a.part_sum = reinterpret_cast<float*>(a.arrivals + (a.ntiles + 1 + 3) / 4 * 4);
  a.part_max = a.part_sum + (int64_t)a.nblocks * d->img_seq;
  a.col_sum = a.part_max + (int64_t)a.nblocks * d->img_seq;
  a.col_max = a.col_sum + d->img_seq;
  a.tile_sums = a.col_max + d->img_seq;
  a.out_idx = d->out_idx; a.out_count = d->out_count;
  cudaStream_t st = as_stream(stream);
  switch (d->dtype) {
    case MSKV_DT_F32:
      return d->round_f16 ? launch_filter<float, kStageF16>(a, st) : launch_filter<float, kStageF32>(a, st);
    case MSKV_DT_F16: return launch_filter<__half, kStageF16>(a, st);
    case MSKV_DT_BF16: return launch_filter<__nv_bfloat16, kStageBF16>(a, st);
    default: return fail(MSKV_ERR_DTYPE, "mskv_image_filter: dtype must be f32, f16 or bf16");
  }
}
