// Library plumbing of libmserve_kv: last-error text, launch counter, pinned mapped host memory.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"

namespace mskv {

std::atomic<uint64_t> g_launches{0};
static thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MSKV_OK;
  return fail(MSKV_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int ensure_smem_limit(const void* kernel, int bytes, const char* what) {
  static std::mutex mu;
  static std::unordered_map<const void*, uint64_t> done;  // bit d: set on device d
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, what);
  const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0;  // devices beyond 63: set every call
  {
    std::lock_guard<std::mutex> g(mu);
    if (bit && (done[kernel] & bit)) return MSKV_OK;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, what);
  }
  std::lock_guard<std::mutex> g(mu);
  done[kernel] |= bit;
  return MSKV_OK;
}

int after_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, what);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MSKV_OK;
}

int check_rows(const mskv_rows& r, const char* side, bool need_v) {
  if (!r.base_k) return fail(MSKV_ERR_ARG, "%s: base_k is NULL", side);
  if (need_v && !r.base_v) return fail(MSKV_ERR_ARG, "%s: base_v is NULL", side);
  if (!r.len && r.len_scalar < 0) return fail(MSKV_ERR_ARG, "%s: negative len_scalar", side);
  if (r.page_table) {
    if (r.page_size <= 0) return fail(MSKV_ERR_ARG, "%s: page_size must be > 0", side);
    if (r.num_pages <= 0) return fail(MSKV_ERR_ARG, "%s: num_pages must be > 0 for a paged side", side);
    if (r.ring_start) return fail(MSKV_ERR_ARG, "%s: a paged side cannot also be a ring", side);
  }
  if (r.ring_start && r.ring_cap <= 0) return fail(MSKV_ERR_ARG, "%s: ring_cap must be > 0", side);
  return MSKV_OK;
}

}  // namespace mskv

using namespace mskv;

extern "C" {

int mskv_abi_version(void) { return MSKV_ABI_VERSION; }

const char* mskv_last_error(void) { return t_last_error.c_str(); }

uint64_t mskv_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int mskv_host_alloc(void** host_ptr, uint64_t bytes) {
  if (!host_ptr) return fail(MSKV_ERR_ARG, "mskv_host_alloc: host_ptr is NULL");
  *host_ptr = nullptr;
  if (bytes == 0) return fail(MSKV_ERR_ARG, "mskv_host_alloc: zero bytes");
  cudaError_t e = cudaHostAlloc(host_ptr, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
  return cuda_status(e, "cudaHostAlloc");
}

int mskv_host_free(void* host_ptr) {
  if (!host_ptr) return MSKV_OK;
  return cuda_status(cudaFreeHost(host_ptr), "cudaFreeHost");
}

int mskv_host_register(void* ptr, uint64_t bytes) {
  if (!ptr || bytes == 0) return fail(MSKV_ERR_ARG, "mskv_host_register: empty range");
  return cuda_status(cudaHostRegister(ptr, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable),
                     "cudaHostRegister");
}

int mskv_host_unregister(void* ptr) {
  if (!ptr) return MSKV_OK;
  return cuda_status(cudaHostUnregister(ptr), "cudaHostUnregister");
}

int mskv_device_view(const void* ptr, void** dev_ptr) {
  if (!dev_ptr) return fail(MSKV_ERR_ARG, "mskv_device_view: dev_ptr is NULL");
  *dev_ptr = nullptr;
  if (!ptr) return fail(MSKV_ERR_ARG, "mskv_device_view: NULL pointer");
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaPointerGetAttributes");
  }
  switch (a.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      *dev_ptr = const_cast<void*>(ptr);
      return MSKV_OK;
    case cudaMemoryTypeHost:
      if (!a.devicePointer)
        return fail(MSKV_ERR_NOT_MAPPED, "pinned host memory %p is not mapped for device access", ptr);
      *dev_ptr = a.devicePointer;
      return MSKV_OK;
    default:
      return fail(MSKV_ERR_NOT_MAPPED, "host memory %p is not pinned (pageable memory cannot be read by the GPU)", ptr);
  }
}

}  // extern "C"
