// Shared helpers of libmserve_kv: error reporting, launch accounting, vector types.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "mserve_kv.h"

namespace mskv {

// Records a formatted message as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Checks cudaGetLastError() after a launch, counts the launch on success.
int after_launch(const char* what);
// Sets a message for a CUDA error and returns MSKV_ERR_CUDA (or MSKV_OK for cudaSuccess).
int cuda_status(cudaError_t e, const char* what);
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device, once per
// (kernel, device) in the process (the attribute is per device).  Thread-safe.
int ensure_smem_limit(const void* kernel, int bytes, const char* what);

extern std::atomic<uint64_t> g_launches;

// Peers a kernel can write to directly (one node: up to 8 GPUs, so 7 others).
constexpr int kMaxPeers = 7;

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch (sm_90 and later).  A kernel started with launch_dependent()
// may become resident while the kernel before it in the stream is still running; it executes
// wait_for_previous_grid() before touching any global memory, which returns once that kernel
// has completed and its writes are visible.  The earlier kernel lets its dependents start
// with allow_dependents() (without it they start when it exits).  Both are hardware
// instructions; neither spins in software.
__device__ __forceinline__ void wait_for_previous_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Params, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                    Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// 1-D bulk copies (cp.async.bulk, never with cluster multicast) completing on an mbarrier in
// shared memory, shared by the row mover and the score kernel.  Every wait is bounded: after
// kBulkWaitIters polls bulk_wait returns false and the caller records MSKV_STATUS_TIMEOUT.
constexpr int kBulkWaitIters = 1 << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool bulk_wait(uint32_t bar, uint32_t parity) {
  for (int it = 0; it < kBulkWaitIters; ++it) {
    uint32_t done;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    if (done) return true;
  }
  return false;
}

// global (or mapped host) -> this CTA's shared memory; src, dst and bytes multiples of 16
__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst_smem), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src_smem), "r"(bytes)
               : "memory");
}

inline int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Byte-vector types used by the row copies.
template <int N> struct Vec;
template <> struct Vec<1> { using T = uint8_t; };
template <> struct Vec<2> { using T = uint16_t; };
template <> struct Vec<4> { using T = uint32_t; };
template <> struct Vec<8> { using T = uint2; };
template <> struct Vec<16> { using T = uint4; };

// Per-segment row addressing shared by the gather, copy and score kernels (mskv_rows).
struct RowsDev {
  const char* base_k;
  const char* base_v;
  int64_t sb, sh, st, sp, pt_stride;
  int64_t len_scalar;
  int64_t num_pages;
  const int32_t* page_table;
  const int32_t* ring_start;
  const int32_t* tok0;
  const int32_t* len;
  int32_t page_size;
  int32_t ring_cap;
};

inline RowsDev to_dev(const mskv_rows& r) {
  RowsDev d;
  d.base_k = static_cast<const char*>(r.base_k);
  d.base_v = static_cast<const char*>(r.base_v);
  d.sb = r.stride_b; d.sh = r.stride_h; d.st = r.stride_t; d.sp = r.stride_page;
  d.pt_stride = r.pt_stride_b; d.len_scalar = r.len_scalar; d.num_pages = r.num_pages;
  d.page_table = r.page_table; d.ring_start = r.ring_start; d.tok0 = r.tok0; d.len = r.len;
  d.page_size = r.page_size; d.ring_cap = r.ring_cap;
  return d;
}

__device__ __forceinline__ int64_t rows_len(const RowsDev& r, int b) {
  return r.len ? (int64_t)r.len[b] : r.len_scalar;
}

// Byte offset of logical token t of segment (b,h), or -1 (with *why set) when the token is
// outside [0, len[b]) or its page is unmapped.
__device__ __forceinline__ int64_t rows_offset(const RowsDev& r, int b, int h, int64_t t,
                                               uint32_t* why, uint32_t oob_bit) {
  if (t < 0 || t >= rows_len(r, b)) { *why |= oob_bit; return -1; }
  if (r.page_table) {
    const int64_t pidx = t / r.page_size;
    const int32_t page = r.page_table[(int64_t)b * r.pt_stride + pidx];
    if (page < 0 || page >= r.num_pages) { *why |= MSKV_STATUS_BAD_PAGE; return -1; }
    return (int64_t)page * r.sp + (int64_t)h * r.sh + (t - pidx * r.page_size) * r.st;
  }
  int64_t p = t;
  if (r.ring_start) {
    p += r.ring_start[b];
    if (p >= r.ring_cap) p -= r.ring_cap;
    if (p < 0 || p >= r.ring_cap) { *why |= oob_bit; return -1; }
  }
  return (int64_t)b * r.sb + (int64_t)h * r.sh + p * r.st;
}

// Host-side sanity checks of an mskv_rows description.
int check_rows(const mskv_rows& r, const char* side, bool need_v);

}  // namespace mskv
