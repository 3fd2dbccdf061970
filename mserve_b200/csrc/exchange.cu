// Peer memory and flags for exchanging score rows between the GPUs of one node without a
// collective library (mskv_ipc_*, mskv_flag_signal, mskv_flag_wait).
//
// The shared selection (one index set per sequence from the scores of every KV head,
// qwen-eljrte/Qwen_Transformer/attention.py:558-572) needs each rank's score rows on every
// rank.  With mskv_score_fanout the score kernel stores each row into every rank's copy as it
// computes it, through CUDA IPC mappings of the peers' buffers (plain stores over NVLink;
// nothing here uses multicast).  Ordering between the GPUs is by epoch-valued flags:
//  * mskv_flag_signal: one thread per rank stores `value` at flags[r][index] with release
//    semantics at system scope, after the kernels before it on the stream completed (their
//    writes were made system-visible before they exited);
//  * mskv_flag_wait: one thread per flag polls it with acquire semantics at system scope until
//    it holds `value` (or at least `value`), sleeping between polls.  The wait is bounded by a
//    time limit read from the global timer; on expiry it sets MSKV_STATUS_TIMEOUT in the
//    status word and returns, so a rank that never signals yields an error on the host, not a
//    hung GPU.
// Each rank's waits only ever wait on kernels of other GPUs (or on earlier kernels of its own
// stream, already complete), never on a kernel that shares its GPU.
#include "common.cuh"

namespace mskv {

__device__ __forceinline__ void store_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ int64_t load_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct SignalArgs {
  int64_t* flags[kMaxPeers + 1];
  int32_t nranks, index;
  int64_t value;
};

// Both flag kernels are launched programmatically dependent on the kernel before them (so
// their launch overlaps its tail) and begin with the hardware grid-dependency wait: they touch
// no flag before that kernel has completed, so a wait never spins beside another kernel of
// this GPU that it depends on.
__global__ void flag_signal_kernel(const SignalArgs a) {
  wait_for_previous_grid();
  __threadfence_system();
  const int r = threadIdx.x;
  if (r < a.nranks) store_release_sys(a.flags[r] + a.index, a.value);
}

__global__ void flag_wait_kernel(const int64_t* flags, int count, int64_t value, int at_least, uint64_t timeout_ns,
                                 uint32_t* status) {
  wait_for_previous_grid();
  const int i = threadIdx.x;
  if (i < count) {
    const uint64_t t0 = global_ns();
    for (;;) {
      const int64_t v = load_acquire_sys(flags + i);
      if (at_least ? v >= value : v == value) break;
      if (global_ns() - t0 > timeout_ns) {
        if (status) atomicOr(status, MSKV_STATUS_TIMEOUT);
        break;
      }
      __nanosleep(256);
    }
  }
  __threadfence();
  allow_dependents();
}

}  // namespace mskv

using namespace mskv;

extern "C" int mskv_ipc_alloc(uint64_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(MSKV_ERR_ARG, "mskv_ipc_alloc: NULL pointer or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_status(e, "mskv_ipc_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "mskv_ipc_alloc");
  }
  *ptr = p;
  return MSKV_OK;
}

extern "C" int mskv_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(MSKV_ERR_ARG, "mskv_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "mskv_ipc_open");
}

extern "C" int mskv_ipc_close(void* ptr) {
  if (!ptr) return MSKV_OK;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "mskv_ipc_close");
}

extern "C" int mskv_ipc_free(void* ptr) {
  if (!ptr) return MSKV_OK;
  return cuda_status(cudaFree(ptr), "mskv_ipc_free");
}

extern "C" uint64_t mskv_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int mskv_flag_signal(int64_t* const* flags, int32_t nranks, int32_t index, int64_t value, void* stream) {
  if (!flags || nranks <= 0 || nranks > kMaxPeers + 1 || index < 0)
    return fail(MSKV_ERR_ARG, "mskv_flag_signal: need 1..%d flag arrays and index >= 0", kMaxPeers + 1);
  SignalArgs a{};
  for (int r = 0; r < nranks; ++r) {
    if (!flags[r]) return fail(MSKV_ERR_ARG, "mskv_flag_signal: NULL flags[%d]", r);
    if ((uintptr_t)flags[r] & 7) return fail(MSKV_ERR_ARG, "mskv_flag_signal: flags[%d] not 8-byte aligned", r);
    a.flags[r] = flags[r];
  }
  a.nranks = nranks;
  a.index = index;
  a.value = value;
  const cudaError_t e = launch_dependent(flag_signal_kernel, dim3(1), dim3(32), 0, as_stream(stream), a);
  if (e != cudaSuccess) return cuda_status(e, "mskv_flag_signal launch");
  return after_launch("mskv_flag_signal");
}

extern "C" int mskv_flag_wait(const int64_t* flags, int32_t count, int64_t value, int32_t at_least,
                              uint64_t timeout_ns, uint32_t* status, void* stream) {
  if (!flags || count <= 0 || count > 1024) return fail(MSKV_ERR_ARG, "mskv_flag_wait: need 1..1024 flags");
  if ((uintptr_t)flags & 7) return fail(MSKV_ERR_ARG, "mskv_flag_wait: flags not 8-byte aligned");
  if (timeout_ns == 0 || timeout_ns > 60ull * 1000000000ull)
    return fail(MSKV_ERR_ARG, "mskv_flag_wait: timeout must lie in (0, 60 s]");
  const int threads = (count + 31) / 32 * 32;
  const cudaError_t e = launch_dependent(flag_wait_kernel, dim3(1), dim3(threads), 0, as_stream(stream), flags,
                                         count, value, at_least, timeout_ns, status);
  if (e != cudaSuccess) return cuda_status(e, "mskv_flag_wait launch");
  return after_launch("mskv_flag_wait");
}
