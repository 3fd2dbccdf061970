// cuda_uva: the torch extension module that MServe's callers import by name
// (qwen-eljrte/Qwen_Transformer/kv_cache.py:511-515, qwen-eljrte/benchmark_kv_transfer.py:36-43;
// the name is fixed by qwen-eljrte/setup_cuda_uva.py:18).  A thin binding: argument checks on
// ATen tensors, output allocation through torch's caching allocator, and one call into the C ABI
// of libmserve_kv (mskv_uva_gather, include/mserve_kv.h) on torch's current CUDA stream.
//
// uva_gather keeps the reference binding's signature, output layout and error texts
// (qwen-eljrte/cuda_uva_kernel.cpp:48-113; qwen-eljrte/cuda_uva_kernel_v2.cpp:86-133).
// Deliberate supersets of its behaviour:
//  * no device synchronisation; the gather is enqueued on the current stream (v1 used the
//    legacy default stream, v2 ends with cudaDeviceSynchronize);
//  * indices may also be a CUDA tensor (the reference requires CPU indices and dereferences
//    that host list from the device, cuda_uva_kernel.cpp:36, 62);
//  * CPU indices are bounds-checked before the launch; CUDA indices on the device (the row is
//    zero-filled and check_errors() raises);
//  * fp8 e4m3 / e5m2 KV (the copy is bitwise);
//  * 64-bit offsets (the reference computes offsets in int, cuda_uva_kernel.cpp:24-40).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDACachingAllocator.h>

#include <mutex>
#include <unordered_map>

#include "mserve_kv.h"

namespace {

std::mutex g_status_mu;
std::unordered_map<int, at::Tensor> g_status;   // device index -> int32 [1] status word

at::Tensor status_word(int device) {
  std::lock_guard<std::mutex> lock(g_status_mu);
  auto it = g_status.find(device);
  if (it != g_status.end()) return it->second;
  at::Tensor w = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  g_status.emplace(device, w);
  return w;
}

bool gather_dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat: case at::kDouble: case at::kHalf: case at::kBFloat16:
    case at::kFloat8_e4m3fn: case at::kFloat8_e5m2:
      return true;
    default:
      return false;
  }
}

void check_input(const at::Tensor& t, const char* name) {
  if (t.is_cuda()) return;
  TORCH_CHECK(t.is_pinned(), name, " must be pinned memory for UVA");
  TORCH_CHECK(t.is_cpu(), name, " must be on CPU (pinned)");
}

}  // namespace

std::vector<at::Tensor> uva_gather(at::Tensor k_in, at::Tensor v_in, at::Tensor indices, int64_t batch_size,
                                   int64_t num_heads, int64_t seq_len, int64_t head_dim) {
  check_input(k_in, "k_in");
  check_input(v_in, "v_in");
  TORCH_CHECK(indices.is_cpu() || indices.is_cuda(), "indices must be on CPU");
  TORCH_CHECK(k_in.scalar_type() == v_in.scalar_type(), "k_in and v_in must have the same dtype");
  TORCH_CHECK(gather_dtype(k_in.scalar_type()), "\"uva_gather\" not implemented for '",
              c10::toString(k_in.scalar_type()), "'");
  TORCH_CHECK(batch_size >= 0 && num_heads >= 0 && seq_len >= 0 && head_dim >= 0, "sizes must be non-negative");
  const int64_t need = batch_size * num_heads * seq_len * head_dim;
  for (const at::Tensor* t : {&k_in, &v_in}) {
    TORCH_CHECK(t->is_contiguous(), (t == &k_in ? "k_in" : "v_in"), " must be contiguous");
    TORCH_CHECK(t->numel() >= need, (t == &k_in ? "k_in" : "v_in"), " has ", t->numel(),
                " elements, fewer than B*H*T*D = ", need);
  }
  TORCH_CHECK(indices.dim() == 1, "indices must be 1-D [num_selected]");
  const int64_t S = indices.size(0);
  const int device = at::cuda::current_device();
  const auto out_opts = k_in.options().device(at::kCUDA, device).pinned_memory(false);
  at::Tensor k_out = at::empty({batch_size, num_heads, S, head_dim}, out_opts);
  at::Tensor v_out = at::empty({batch_size, num_heads, S, head_dim}, out_opts);
  if (S == 0 || batch_size * num_heads * head_dim == 0) return {k_out, v_out};

  at::cuda::CUDAStream stream = at::cuda::getCurrentCUDAStream(device);
  at::Tensor idx;
  if (indices.is_cuda()) {
    idx = indices.to(at::TensorOptions().device(at::kCUDA, device).dtype(at::kLong)).contiguous();
  } else {
    at::Tensor i64 = indices.to(at::kLong).contiguous();
    const int64_t lo = i64.min().item<int64_t>(), hi = i64.max().item<int64_t>();
    TORCH_CHECK(lo >= 0 && hi < seq_len, "indices out of range [0, ", seq_len, "): min ", lo, ", max ", hi);
    // Asynchronous H2D from page-locked memory (torch's pinned host allocator keeps the block
    // until the copy has run), so the call never waits for earlier work on the stream.
    if (!i64.is_pinned()) i64 = i64.pin_memory();
    idx = i64.to(at::TensorOptions().device(at::kCUDA, device), /*non_blocking=*/true);
  }
  at::Tensor status = status_word(device);
  const int rc = mskv_uva_gather(k_in.data_ptr(), v_in.data_ptr(), static_cast<const int64_t*>(idx.data_ptr()), S,
                                 batch_size, num_heads, seq_len, head_dim, (int32_t)k_in.element_size(),
                                 k_out.data_ptr(), v_out.data_ptr(), static_cast<uint32_t*>(status.data_ptr()),
                                 stream.stream());
  TORCH_CHECK(rc == MSKV_OK, "uva_gather: ", mskv_last_error());
  // the device copy of the indices stays allocated until the gather has run
  c10::cuda::CUDACachingAllocator::recordStream(idx.storage().data_ptr(), stream);
  return {k_out, v_out};
}

void check_errors() {
  const int device = at::cuda::current_device();
  at::Tensor w = status_word(device);
  const int v = w.item<int>();
  if (v) {
    w.zero_();
    TORCH_CHECK(false, "uva_gather: token index out of range (status 0x", std::hex, v, "); the rows were zero-filled");
  }
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "UVA gather of selected KV rows from pinned host memory (libmserve_kv, sm_100a)";
  m.def("uva_gather", &uva_gather, "k_out[b,h,s,:] = k_in[b,h,indices[s],:] (same for v) -> [k_out, v_out]",
        py::arg("k_in"), py::arg("v_in"), py::arg("indices"), py::arg("batch_size"), py::arg("num_heads"),
        py::arg("seq_len"), py::arg("head_dim"));
  m.def("check_errors", &check_errors, "raise if a gather on the current device met an out-of-range CUDA index");
}
