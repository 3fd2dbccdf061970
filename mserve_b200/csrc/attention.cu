// Decode attention over the selected rows (mskv_sparse_attention).
//
// Reference: sparse_sdpa_attention (qwen-eljrte/Qwen_Transformer/attention.py:591-641):
// softmax(q·K_selᵀ/sqrt(D))·V_sel with no mask.  Here K_sel/V_sel keep the KV-head layout
// (no repeat_kv): all G query heads (times q_len query rows) of a KV head are served by one
// pass over that head's selected rows, so every gathered byte is read once from HBM.
//
// Split-sequence ("flash-decoding") schedule, fast path (16-bit, D in {64,128}, G*q_len <= 8
// or 16 for D=64, contiguous rows): CTA (segment, split) owns kTile = 64 selected rows.
//   0. one thread starts two bulk copies (K tile, V tile: contiguous 8-16 KB each) into shared
//      memory on an mbarrier while all threads stage their query slice in registers;
//   1. QKᵀ: a warp serves 32/SL query rows, lane = (query row, 16-byte d-slice); each lane
//      walks the 64 K rows (one 16-byte shared load per row, shared by the warp's query rows)
//      accumulating one partial dot per row, then a butterfly reduce-scatter over the SL
//      slice lanes leaves each lane with the full scores of 64/SL rows;
//   2. tile max / exp / sum per query row with xor-shuffles; probabilities -> shared memory;
//   3. P·V with the same lane mapping: each lane accumulates its 8 output dims directly;
//   4. (m, l, acc) partials -> workspace; the last CTA of the segment (atomic ticket) merges
//      the splits and writes the output, then re-arms the ticket for the next launch.
// Other shapes use a one-warp-per-output-row kernel with an online softmax.
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace mskv {

constexpr int kAtThreads = 128;
constexpr int kAtTile = 64;         // selected rows per CTA
constexpr int kAtWsHeader = 4096;   // bytes reserved for the per-segment tickets (<= 1024 segments)

struct AttnDev {
  const char* q;
  int64_t q_sb, q_sh, q_sq;
  const char* k;
  const char* v;
  int64_t kv_seg, kv_s;
  const int32_t* counts;
  char* out;
  int64_t o_sb, o_sh, o_sq;
  unsigned* tickets;       // [segments]
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

template <bool BF16, int D>
__global__ void __launch_bounds__(kAtThreads) attn_split_kernel(const AttnDev a) {
  constexpr int ROWB = D * 2;
  constexpr int SL = D / 8;            // 16-byte d-slices per row = lanes per query row
  constexpr int RPW = 32 / SL;         // query rows per warp
  constexpr int RPL = kAtTile / SL;    // score rows per lane after the reduce-scatter
  __shared__ __align__(128) uint8_t sK[kAtTile * ROWB];
  __shared__ __align__(128) uint8_t sV[kAtTile * ROWB];
  __shared__ float s_p[4 * RPW][kAtTile];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_last;

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
  const int sl = lane % SL;                 // d-slice
  const int r = warp * RPW + lane / SL;     // query row of this lane
  const bool active = r < nr;

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(nrows * ROWB);
    mbar_arrive_expect_tx(&bar, 2 * bytes);
    if (bytes) {
      bulk_load(sK, a.k + (int64_t)seg * a.kv_seg + (int64_t)r0 * a.kv_s, bytes, &bar);
      bulk_load(sV, a.v + (int64_t)seg * a.kv_seg + (int64_t)r0 * a.kv_s, bytes, &bar);
    }
  }
  // query slice of this lane (pre-scaled), while the copies are in flight
  float qf[8];
  {
    const int g = active ? r / a.q_len : 0, i = active ? r - (r / a.q_len) * a.q_len : 0;
    const char* qp = a.q + (int64_t)b * a.q_sb + (int64_t)(hk * G + g) * a.q_sh + (int64_t)i * a.q_sq;
    const uint4 raw = active ? *reinterpret_cast<const uint4*>(qp + sl * 16) : make_uint4(0, 0, 0, 0);
    cvt8(raw, qf, BF16);
#pragma unroll
    for (int e = 0; e < 8; ++e) qf[e] *= a.scale;
  }
  const bool ok = mbar_wait(&bar, 0, kWaitTimeoutNs);
  if (__syncthreads_or(!ok)) {
    if (tid == 0 && a.status) atomicOr(a.status, MSKV_STATUS_TIMEOUT);
    mbar_wait(&bar, 0, kDrainTimeoutNs);
    return;  // every CTA of the launch reaches this point together only on a broken device
  }

  // 1. scores of the 64 rows for this lane's query row (partial over its d-slice)
  float part[kAtTile];
#pragma unroll
  for (int row = 0; row < kAtTile; ++row) {
    float acc = 0.f;
    if (row < nrows) {
      float f[8];
      cvt8(*reinterpret_cast<const uint4*>(sK + row * ROWB + sl * 16), f, BF16);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(qf[e], f[e], acc);
    }
    part[row] = acc;
  }
  reduce_scatter_n<kAtTile, SL>(part, sl);   // part[0..RPL) = rows [sl*RPL, (sl+1)*RPL)
  // 2. softmax statistics over the tile (rows >= nrows excluded)
  float m = -INFINITY;
#pragma unroll
  for (int x = 0; x < RPL; ++x)
    if (sl * RPL + x < nrows) m = fmaxf(m, part[x]);
#pragma unroll
  for (int o = SL / 2; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float l = 0.f;
#pragma unroll
  for (int x = 0; x < RPL; ++x) {
    const int row = sl * RPL + x;
    const float p = row < nrows ? expf(part[x] - m) : 0.f;
    s_p[warp * RPW + lane / SL][row] = p;
    l += p;
  }
#pragma unroll
  for (int o = SL / 2; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  __syncwarp();
  // 3. P·V for this lane's 8 output dims
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  const float* prow = s_p[warp * RPW + lane / SL];
  for (int row = 0; row < nrows; ++row) {
    float f[8];
    cvt8(*reinterpret_cast<const uint4*>(sV + row * ROWB + sl * 16), f, BF16);
    const float p = prow[row];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(p, f[e], acc[e]);
  }
  // 4. partial -> workspace, last CTA of the segment merges
  const int64_t wstride = (int64_t)a.nr * (D + 2);
  float* wp = a.ws + ((int64_t)seg * a.splits + split) * wstride;
  if (active) {
    float4* dst = reinterpret_cast<float4*>(wp + (int64_t)r * (D + 2) + sl * 8);
    if (((uintptr_t)dst & 15) == 0) {
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) wp[(int64_t)r * (D + 2) + sl * 8 + e] = acc[e];
    }
    if (sl == 0) {
      wp[(int64_t)r * (D + 2) + D] = nrows > 0 ? m : -INFINITY;
      wp[(int64_t)r * (D + 2) + D + 1] = nrows > 0 ? l : 0.f;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&a.tickets[seg], 1u);
    s_last = prev == (unsigned)(a.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (active) {
    const float* base = a.ws + (int64_t)seg * a.splits * wstride + (int64_t)r * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < a.splits; ++s) M = fmaxf(M, __ldcg(base + s * wstride + D));
    float L = 0.f, o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float ms = __ldcg(base + s * wstride + D);
      if (ms == -INFINITY) continue;
      const float w = expf(ms - M);
      L += __ldcg(base + s * wstride + D + 1) * w;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] += __ldcg(base + s * wstride + sl * 8 + e) * w;
    }
    const int g = r / a.q_len, i = r - g * a.q_len;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    T* op = reinterpret_cast<T*>(a.out + (int64_t)b * a.o_sb + (int64_t)(hk * G + g) * a.o_sh + (int64_t)i * a.o_sq);
#pragma unroll
    for (int e = 0; e < 8; ++e) op[sl * 8 + e] = from_f<T>(L > 0.f ? o[e] / L : 0.f);
  }
  if (tid == 0) a.tickets[seg] = 0u;  // re-arm for the next launch on this workspace
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
  const int rows_max = 4 * (32 / (d->head_dim / 8));  // 4 warps x query rows per warp
  if (G * d->q_len > rows_max) return false;
  if (d->kv_stride_s != (int64_t)d->head_dim * 2) return false;  // tiles are single bulk copies
  if ((int64_t)d->batch * d->kv_heads > kAtWsHeader / 4) return false;
  const uint64_t al = (uint64_t)(uintptr_t)d->k | (uint64_t)(uintptr_t)d->v | (uint64_t)d->kv_stride_seg |
                      (uint64_t)(uintptr_t)d->q | (uint64_t)d->q_stride_b | (uint64_t)d->q_stride_h |
                      (uint64_t)d->q_stride_q;
  return (al & 15) == 0;
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
  return (uint64_t)(kAtWsHeader + (int64_t)d->batch * d->kv_heads * splits_of(d) * nr * (d->head_dim + 2) * 4);
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
    a.tickets = static_cast<unsigned*>(d->workspace);
    a.ws = reinterpret_cast<float*>(static_cast<char*>(d->workspace) + kAtWsHeader);
    a.splits = (int)splits_of(d);
    const int64_t blocks = (int64_t)d->batch * d->kv_heads * a.splits;
    if (blocks > 0x7fffffffLL) return fail(MSKV_ERR_RANGE, "mskv_sparse_attention: grid too large");
    const bool bf = d->dtype == MSKV_DT_BF16;
    if (d->head_dim == 128) {
      if (bf) attn_split_kernel<true, 128><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
      else attn_split_kernel<false, 128><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
    } else {
      if (bf) attn_split_kernel<true, 64><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
      else attn_split_kernel<false, 64><<<(unsigned)blocks, kAtThreads, 0, st>>>(a);
    }
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
// device (cudaGetSymbolAddress, on that device's first call) and cached; nothing is
// allocated or freed.  All calls on a device share the array, so calls that overlap on the
// GPU (different streams without ordering) race on it.
static __device__ __align__(256) unsigned char g_attn_scratch[MSKV_NOALLOC_ATTN_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_dev[kMaxDevices] = {};

int scratch_of_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MSKV_ERR_RANGE, "device index %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(attention scratch)");
    g_scratch_dev[dev] = p;
  }
  *out = g_scratch_dev[dev];
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
  if (need > 0) {
    // The per-segment tickets must start at zero; the array keeps whatever the last call
    // (possibly an interrupted one) left there.
    cudaError_t e = cudaMemsetAsync(scratch, 0, kAtWsHeader, as_stream(stream));
    if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(attention scratch tickets)");
  }
  return mskv_sparse_attention(&c, stream);
}
