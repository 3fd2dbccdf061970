// Image-token filter of a prefill attention map (mskv_image_filter).
//
// Replaces dual_attention_filter (qwen-eljrte/Qwen_Transformer/dual_attention_filter.py:6-103):
// from the attention probabilities of batch 0, the block of text rows x image columns
// [H, text, img] is averaged over the heads; per image token the column sum over the text rows
// (the "global" score) and the column maximum (the "individual" score) decide whether it is
// dropped:  drop = sum < total * global_thr  and  max < individual_thr,  total = the sum of
// all column sums.  The kept image tokens are returned in ascending order.
//
// Two kernels, the second launched programmatically dependent on the first:
//  * filter_columns_kernel: one thread per image column, coalesced along the columns; the head
//    mean is accumulated in head order and divided by H, the column sum in text-row order
//    (the reference's reduction order for these outer dimensions), in fp32; each CTA also
//    writes the sum of its columns' sums;
//  * filter_select_kernel: one CTA sums the CTA partials in order, applies the two thresholds
//    and compacts the kept columns in order through bitmaps and a block scan.
#include "common.cuh"

namespace mskv {

struct FilterDev {
  const char* attn;
  int64_t sh, sq, sk;            // element strides of head, query row, key column (batch 0)
  int32_t dtype, heads, txt_beg, text, img_beg, img;
  float global_thr, individual_thr;
  float* col_sum;
  float* col_max;
  float* cta_sums;
  int64_t* out_idx;
  int32_t* out_count;
};

constexpr int kFcThreads = 256;
constexpr int kFsThreads = 1024;

template <typename T> __device__ __forceinline__ float as_f32(T x);
template <> __device__ __forceinline__ float as_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float as_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float as_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__global__ void __launch_bounds__(kFcThreads) filter_columns_kernel(const FilterDev a) {
  allow_dependents();
  __shared__ float s_part[kFcThreads / 32];
  const int j = blockIdx.x * kFcThreads + threadIdx.x;
  float sum = 0.f, mx = -INFINITY;
  if (j < a.img) {
    const T* col = reinterpret_cast<const T*>(a.attn) + (int64_t)(a.img_beg + j) * a.sk;
    for (int i = 0; i < a.text; ++i) {
      const T* p = col + (int64_t)(a.txt_beg + i) * a.sq;
      float hs = 0.f;
      for (int h = 0; h < a.heads; ++h) hs += as_f32<T>(p[(int64_t)h * a.sh]);
      const float hm = hs / (float)a.heads;
      sum += hm;
      mx = fmaxf(mx, hm);
    }
    a.col_sum[j] = sum;
    a.col_max[j] = mx;
  }
  // this CTA's share of the grand total, summed in a fixed order
  float v = j < a.img ? sum : 0.f;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kFcThreads / 32; ++w) t += s_part[w];
    a.cta_sums[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(kFsThreads) filter_select_kernel(const FilterDev a, int nctas) {
  wait_for_previous_grid();  // column sums and maxima come from filter_columns_kernel
  __shared__ float s_total;
  __shared__ uint32_t s_wcnt[kFsThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    float t = 0.f;
    for (int c = 0; c < nctas; ++c) t += a.cta_sums[c];
    s_total = t;
  }
  __syncthreads();
  const float thr = s_total * a.global_thr;
  // ordered compaction: word q covers columns [32q, 32q+32); warp w takes words w, w+32, ...
  // in rounds, the round's 32 words in token order across the warps
  uint32_t base = 0;
  for (int q0 = 0; 32 * q0 < a.img; q0 += kFsThreads / 32) {
    const int q = q0 + warp;
    const int j = 32 * q + lane;
    bool keep = false;
    if (j < a.img) keep = !(a.col_sum[j] < thr && a.col_max[j] < a.individual_thr);
    const uint32_t m = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) s_wcnt[warp] = __popc(m);
    __syncthreads();
    uint32_t before = 0, round = 0;
    for (int w = 0; w < kFsThreads / 32; ++w) {
      const uint32_t c = s_wcnt[w];
      if (w < warp) before += c;
      round += c;
    }
    uint32_t lt;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
    if (keep) a.out_idx[base + before + __popc(m & lt)] = j;
    base += round;
    __syncthreads();   // s_wcnt is rewritten next round
  }
  if (tid == 0) *a.out_count = (int32_t)base;
}

}  // namespace mskv

using namespace mskv;

extern "C" uint64_t mskv_image_filter_workspace_bytes(int32_t img_seq) {
  if (img_seq <= 0) return 0;
  const uint64_t nctas = ((uint64_t)img_seq + kFcThreads - 1) / kFcThreads;
  return (2ull * (uint64_t)img_seq + nctas) * sizeof(float);
}

extern "C" int mskv_image_filter(const mskv_filter_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_image_filter: NULL descriptor");
  if (d->heads <= 0 || d->text_seq <= 0 || d->img_seq < 0 || d->img_start < 0 || d->text_start < 0)
    return fail(MSKV_ERR_ARG, "mskv_image_filter: bad sizes (heads and text_seq must be positive)");
  if (!d->attn || !d->out_idx || !d->out_count) return fail(MSKV_ERR_ARG, "mskv_image_filter: NULL pointer");
  if (d->img_seq > 0 && (!d->workspace || d->workspace_bytes < mskv_image_filter_workspace_bytes(d->img_seq)))
    return fail(MSKV_ERR_ARG, "mskv_image_filter: workspace needs %llu bytes",
                (unsigned long long)mskv_image_filter_workspace_bytes(d->img_seq));
  if (((uintptr_t)d->workspace & 3) != 0) return fail(MSKV_ERR_ARG, "mskv_image_filter: workspace must be 4-byte aligned");
  FilterDev a{};
  a.attn = static_cast<const char*>(d->attn);
  a.sh = d->stride_h; a.sq = d->stride_q; a.sk = d->stride_k;
  a.dtype = d->dtype; a.heads = d->heads; a.text = d->text_seq; a.img = d->img_seq;
  a.img_beg = d->img_start; a.txt_beg = d->text_start;
  a.global_thr = d->global_thr; a.individual_thr = d->individual_thr;
  a.col_sum = static_cast<float*>(d->workspace);
  a.col_max = a.col_sum + d->img_seq;
  a.cta_sums = a.col_max + d->img_seq;
  a.out_idx = d->out_idx; a.out_count = d->out_count;
  cudaStream_t st = as_stream(stream);
  const int nctas = (d->img_seq + kFcThreads - 1) / kFcThreads;
  if (d->img_seq > 0) {
    switch (d->dtype) {
      case MSKV_DT_F32: filter_columns_kernel<float><<<nctas, kFcThreads, 0, st>>>(a); break;
      case MSKV_DT_F16: filter_columns_kernel<__half><<<nctas, kFcThreads, 0, st>>>(a); break;
      case MSKV_DT_BF16: filter_columns_kernel<__nv_bfloat16><<<nctas, kFcThreads, 0, st>>>(a); break;
      default: return fail(MSKV_ERR_DTYPE, "mskv_image_filter: dtype must be f32, f16 or bf16");
    }
    int rc = after_launch("mskv_image_filter");
    if (rc) return rc;
  }
  const cudaError_t e = launch_dependent(filter_select_kernel, dim3(1), dim3(kFsThreads), 0, st, a, nctas);
  if (e != cudaSuccess) return cuda_status(e, "mskv_image_filter launch");
  return after_launch("mskv_image_filter");
}
