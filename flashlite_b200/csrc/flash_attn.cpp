// Torch binding of libflashlite_b200: the drop-in for the reference's pybind11
// module `flash_attn_wmma` (thebigblender/FlashLite csrc/flash_attn.cpp:4-29).
//
// This file only validates torch tensors, applies the reference's argument
// conventions and calls the C ABI (include/flashlite_b200.h); it contains no
// kernels and links no CUDA code of its own. Error messages of the checks are
// the reference's (csrc/kernel_flash2.cu:741-764, csrc/kernel_naive.cu:252-276)
// so callers that match on them keep working.

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <optional>
#include <string>
#include <vector>

#include "../../include/flashlite_b200.h"

namespace {

void check_status(int status) {
  TORCH_CHECK(status == FL_OK, "flashlite_b200: ", fl_status_str(status), ": ", fl_last_error());
}

void* stream_of(const torch::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// flash_attn::flash_attn_forward_flash2 (csrc/kernel_flash2.cu:732-839)
torch::Tensor forward_flash2(torch::Tensor q, torch::Tensor k, torch::Tensor v, double sm_scale,
                             bool is_causal, std::optional<torch::Tensor> out) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "All tensors must be on CUDA");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "All tensors must be contiguous");
  TORCH_CHECK(q.dtype() == torch::kHalf && k.dtype() == torch::kHalf && v.dtype() == torch::kHalf,
              "All tensors must be FP16 (Half)");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "Tensors must be 4D [B, H, N, D]");
  const int64_t B = q.size(0), H = q.size(1), N = q.size(2), D = q.size(3);
  TORCH_CHECK(k.size(0) == B && k.size(1) == H && k.size(3) == D,
              "Key dimensions must match Query dimensions [B, H, N_k, D]");
  TORCH_CHECK(v.size(0) == B && v.size(1) == H && v.size(2) == k.size(2) && v.size(3) == D,
              "Value dimensions must match Key dimensions [B, H, N_k, D]");
  TORCH_CHECK(D == 64, "FlashLite WMMA kernel currently requires head_dim == 64");
  // The reference assumes N_k == N_q without checking it (its kernels bound
  // K/V reads by the query length); here the assumption is enforced.
  TORCH_CHECK(k.size(2) == N, "forward_flash2 requires N_k == N_q");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "All tensors must be on the same CUDA device");

  torch::Tensor out_tensor;
  if (out.has_value() && out.value().defined()) {
    out_tensor = out.value();
    TORCH_CHECK(out_tensor.is_cuda() && out_tensor.is_contiguous(),
                "out tensor must be contiguous CUDA tensor");
    TORCH_CHECK(out_tensor.sizes() == q.sizes(), "out tensor shape must match q");
    TORCH_CHECK(out_tensor.dtype() == torch::kHalf, "out tensor dtype must be FP16");
    TORCH_CHECK(out_tensor.device() == q.device(), "out tensor must be on the same device as q");
  } else {
    out_tensor = torch::empty_like(q);
  }
  if (out_tensor.numel() == 0) return out_tensor;
  const c10::cuda::CUDAGuard guard(q.device());
  // sm_scale == 0 -> 1/sqrt(D) is applied by the C ABI (csrc/kernel_flash2.cu:769-771)
  void* const stream = stream_of(q);
  int status;
  {
    // The launch blocks while the device's launch queue is full; other
    // Python threads keep running meanwhile (the error text is thread-local).
    pybind11::gil_scoped_release no_gil;
    status = fl_flash2_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out_tensor.data_ptr(), B, H, N,
                           D, static_cast<float>(sm_scale), is_causal ? 1 : 0, stream);
  }
  check_status(status);
  return out_tensor;
}

// flash_attn::flash_attn_forward_naive (csrc/kernel_naive.cu:242-323)
torch::Tensor forward_naive(torch::Tensor q, torch::Tensor k, torch::Tensor v, double sm_scale,
                            bool is_causal) {
  TORCH_CHECK(q.is_cuda(), "Query tensor must be on CUDA");
  TORCH_CHECK(k.is_cuda(), "Key tensor must be on CUDA");
  TORCH_CHECK(v.is_cuda(), "Value tensor must be on CUDA");
  TORCH_CHECK(q.is_contiguous(), "Query tensor must be contiguous");
  TORCH_CHECK(k.is_contiguous(), "Key tensor must be contiguous");
  TORCH_CHECK(v.is_contiguous(), "Value tensor must be contiguous");
  TORCH_CHECK(q.dtype() == torch::kHalf, "Query tensor must be FP16 (Half)");
  TORCH_CHECK(k.dtype() == torch::kHalf, "Key tensor must be FP16 (Half)");
  TORCH_CHECK(v.dtype() == torch::kHalf, "Value tensor must be FP16 (Half)");
  TORCH_CHECK(q.dim() == 4, "Query tensor must have 4 dimensions [B, H, N, D]");
  TORCH_CHECK(k.dim() == 4, "Key tensor must have 4 dimensions [B, H, N, D]");
  TORCH_CHECK(v.dim() == 4, "Value tensor must have 4 dimensions [B, H, N, D]");
  const int64_t B = q.size(0), H = q.size(1), N = q.size(2), D = q.size(3);
  TORCH_CHECK(k.size(0) == B && k.size(1) == H && k.size(3) == D,
              "Key dimensions must match Query dimensions [B, H, N_k, D]");
  TORCH_CHECK(v.size(0) == B && v.size(1) == H && v.size(2) == k.size(2) && v.size(3) == D,
              "Value dimensions must match Key dimensions [B, H, N_k, D]");
  TORCH_CHECK(k.size(2) == N, "forward_naive requires N_k == N_q");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "All tensors must be on the same CUDA device");
  auto out = torch::empty_like(q);
  if (out.numel() == 0) return out;
  const c10::cuda::CUDAGuard guard(q.device());
  check_status(fl_naive_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, N, D,
                            static_cast<float>(sm_scale), is_causal ? 1 : 0, stream_of(q)));
  return out;
}

// Extension without a reference counterpart: N_k != N_q, position offsets,
// optional LSE output (fl_flash2_fwd_ex). Returns (out, lse); lse is an
// empty tensor unless return_lse.
std::vector<torch::Tensor> forward_flash2_ex(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                             double sm_scale, bool is_causal, int64_t q_offset,
                                             int64_t kv_offset, std::optional<torch::Tensor> out,
                                             bool return_lse, std::string layout) {
  TORCH_CHECK(layout == "bhnd" || layout == "bnhd", "layout must be 'bhnd' or 'bnhd'");
  const bool bnhd = layout == "bnhd";
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "All tensors must be on CUDA");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "All tensors must be contiguous");
  TORCH_CHECK(q.dtype() == torch::kHalf && k.dtype() == torch::kHalf && v.dtype() == torch::kHalf,
              "All tensors must be FP16 (Half)");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4,
              bnhd ? "Tensors must be 4D [B, N, H, D]" : "Tensors must be 4D [B, H, N, D]");
  const int hd = bnhd ? 2 : 1, nd = bnhd ? 1 : 2;  // dimension of heads / rows
  const int64_t B = q.size(0), H = q.size(hd), Nq = q.size(nd), D = q.size(3), Nk = k.size(nd);
  TORCH_CHECK(k.size(0) == B && k.size(hd) == H && k.size(3) == D,
              bnhd ? "Key dimensions must match Query dimensions [B, N_k, H, D]"
                   : "Key dimensions must match Query dimensions [B, H, N_k, D]");
  TORCH_CHECK(v.sizes() == k.sizes(), "Value dimensions must match Key dimensions [B, H, N_k, D]");
  TORCH_CHECK(D == 64 || D == 128, "forward_flash2_ex requires head_dim 64 or 128");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "All tensors must be on the same CUDA device");
  torch::Tensor out_tensor;
  if (out.has_value() && out.value().defined()) {
    out_tensor = out.value();
    TORCH_CHECK(out_tensor.is_cuda() && out_tensor.is_contiguous(),
                "out tensor must be contiguous CUDA tensor");
    TORCH_CHECK(out_tensor.sizes() == q.sizes(), "out tensor shape must match q");
    TORCH_CHECK(out_tensor.dtype() == torch::kHalf, "out tensor dtype must be FP16");
    TORCH_CHECK(out_tensor.device() == q.device(), "out tensor must be on the same device as q");
  } else {
    out_tensor = torch::empty_like(q);
  }
  torch::Tensor lse = return_lse ? torch::empty({B, H, Nq}, q.options().dtype(torch::kFloat32))
                                 : torch::empty({0}, q.options().dtype(torch::kFloat32));
  if (out_tensor.numel() == 0) return {out_tensor, lse};
  const c10::cuda::CUDAGuard guard(q.device());
  check_status(fl_flash2_fwd_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), out_tensor.data_ptr(),
                                return_lse ? lse.data_ptr<float>() : nullptr, B, H, Nq, Nk, D,
                                q_offset, kv_offset, static_cast<float>(sm_scale), is_causal ? 1 : 0,
                                bnhd ? FL_LAYOUT_BNHD : FL_LAYOUT_BHND, stream_of(q)));
  return {out_tensor, lse};
}

// One ring-attention block step (no reference counterpart): merges
// attention of q [B,H,Nq,64] against k/v [B,H,Nk,64] into (o_acc fp32
// [B,H,Nq,64], lse fp32 [B,H,Nq]).
void forward_block(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o_acc,
                   torch::Tensor lse, int64_t q_offset, int64_t kv_offset, double sm_scale,
                   bool is_causal, bool first) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && o_acc.is_cuda() && lse.is_cuda(),
              "All tensors must be on CUDA");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() &&
                  o_acc.is_contiguous() && lse.is_contiguous(),
              "All tensors must be contiguous");
  TORCH_CHECK(q.dtype() == torch::kHalf && k.dtype() == torch::kHalf && v.dtype() == torch::kHalf,
              "q, k, v must be FP16 (Half)");
  TORCH_CHECK(o_acc.dtype() == torch::kFloat && lse.dtype() == torch::kFloat,
              "o_acc and lse must be float32");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "Tensors must be 4D [B, H, N, D]");
  const int64_t B = q.size(0), H = q.size(1), Nq = q.size(2), D = q.size(3);
  TORCH_CHECK(k.size(0) == B && k.size(1) == H && k.size(3) == D && v.sizes() == k.sizes(),
              "Key/Value dimensions must be [B, H, N_k, D]");
  TORCH_CHECK(o_acc.sizes() == q.sizes(), "o_acc shape must match q");
  TORCH_CHECK(lse.numel() == B * H * Nq, "lse must hold B*H*Nq values");
  const c10::cuda::CUDAGuard guard(q.device());
  check_status(fl_flash2_fwd_block(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                   o_acc.data_ptr<float>(), lse.data_ptr<float>(), B * H, Nq,
                                   k.size(2), D, q_offset, kv_offset, static_cast<float>(sm_scale),
                                   is_causal ? 1 : 0, first ? 1 : 0, stream_of(q)));
}

void ring_finalize(torch::Tensor o_acc, torch::Tensor out) {
  TORCH_CHECK(o_acc.is_cuda() && out.is_cuda(), "All tensors must be on CUDA");
  TORCH_CHECK(o_acc.is_contiguous() && out.is_contiguous(), "All tensors must be contiguous");
  TORCH_CHECK(o_acc.dtype() == torch::kFloat && out.dtype() == torch::kHalf,
              "o_acc must be float32 and out FP16");
  TORCH_CHECK(o_acc.numel() == out.numel(), "o_acc and out must have the same size");
  const c10::cuda::CUDAGuard guard(out.device());
  check_status(fl_ring_finalize(o_acc.data_ptr<float>(), out.data_ptr(), out.numel(), stream_of(out)));
}

// Synchronises the current stream and returns the device error bits raised by
// kernels since the last call (0 = none); clears them.
int64_t device_error() {
  uint32_t flags = 0;
  const int st = fl_device_error(
      static_cast<void*>(c10::cuda::getCurrentCUDAStream().stream()), &flags);
  TORCH_CHECK(st == FL_OK || st == FL_ERR_DEVICE_TIMEOUT, "flashlite_b200: ", fl_status_str(st),
              ": ", fl_last_error());
  return static_cast<int64_t>(flags);
}

// FA2 backward (no reference counterpart): gradients of
// softmax(sm_scale * q k^T) v given the forward output `out`, its gradient
// `dout` and the forward's LSE (forward_flash2_ex(..., return_lse=True));
// layout "bnhd" takes [B, N, H, D] tensors (lse stays [B, H, N]).
// Returns (dq, dk, dv); the fp32 workspace is a torch allocation.
std::vector<torch::Tensor> backward_flash2(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                           torch::Tensor out, torch::Tensor dout, torch::Tensor lse,
                                           double sm_scale, bool is_causal, std::string layout) {
  TORCH_CHECK(layout == "bhnd" || layout == "bnhd", "layout must be 'bhnd' or 'bnhd'");
  const bool bnhd = layout == "bnhd";
  for (const torch::Tensor* t : {&q, &k, &v, &out, &dout}) {
    TORCH_CHECK(t->is_cuda(), "All tensors must be on CUDA");
    TORCH_CHECK(t->is_contiguous(), "All tensors must be contiguous");
    TORCH_CHECK(t->dtype() == torch::kHalf, "q, k, v, out and dout must be FP16 (Half)");
    TORCH_CHECK(t->dim() == 4, bnhd ? "Tensors must be 4D [B, N, H, D]" : "Tensors must be 4D [B, H, N, D]");
    TORCH_CHECK(t->sizes() == q.sizes(), "q, k, v, out and dout must have the same shape");
    TORCH_CHECK(t->device() == q.device(), "All tensors must be on the same CUDA device");
  }
  const int64_t B = q.size(0), H = q.size(bnhd ? 2 : 1), N = q.size(bnhd ? 1 : 2), D = q.size(3);
  TORCH_CHECK(D == 64, "backward_flash2 requires head_dim == 64");
  TORCH_CHECK(lse.is_cuda() && lse.is_contiguous() && lse.dtype() == torch::kFloat &&
                  lse.device() == q.device(),
              "lse must be a contiguous float32 CUDA tensor on q's device");
  TORCH_CHECK(lse.numel() == B * H * N, "lse must hold B*H*N values [B, H, N]");
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  if (q.numel() == 0) return {dq, dk, dv};
  const c10::cuda::CUDAGuard guard(q.device());
  const size_t ws_bytes = fl_flash2_bwd_workspace_size(B, H, N, D);
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, q.options().dtype(torch::kUInt8));
  check_status(fl_flash2_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
                             lse.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                             ws.data_ptr(), ws_bytes, B, H, N, D, static_cast<float>(sm_scale),
                             is_causal ? 1 : 0, bnhd ? FL_LAYOUT_BNHD : FL_LAYOUT_BHND, stream_of(q)));
  return {dq, dk, dv};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "FlashAttention-2 forward for B200 (sm_100a): tcgen05 + TMA + TMEM";
  m.def("forward_naive", &forward_naive, "Naive attention forward (CUDA-core baseline)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("sm_scale") = 0.0,
        py::arg("is_causal") = false);
  m.def("forward_flash2", &forward_flash2, "FlashAttention-2 forward (tcgen05, sm_100a)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("sm_scale") = 0.0,
        py::arg("is_causal") = false, py::arg("out") = py::none());
  m.def("forward_flash2_ex", &forward_flash2_ex,
        "FA2 forward with N_k != N_q, position offsets and optional LSE; returns (out, lse)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("sm_scale") = 0.0,
        py::arg("is_causal") = false, py::arg("q_offset") = 0, py::arg("kv_offset") = 0,
        py::arg("out") = py::none(), py::arg("return_lse") = false, py::arg("layout") = "bhnd");
  m.def("forward_block", &forward_block, "Ring-attention block step with LSE merge",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o_acc"), py::arg("lse"),
        py::arg("q_offset"), py::arg("kv_offset"), py::arg("sm_scale") = 0.0,
        py::arg("is_causal") = true, py::arg("first") = false);
  m.def("ring_finalize", &ring_finalize, "Cast the merged fp32 ring output to fp16",
        py::arg("o_acc"), py::arg("out"));
  m.def("backward_flash2", &backward_flash2,
        "FA2 backward (tcgen05, sm_100a); returns (dq, dk, dv)", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("out"), py::arg("dout"), py::arg("lse"), py::arg("sm_scale") = 0.0,
        py::arg("is_causal") = false, py::arg("layout") = "bhnd");
  m.def("device_error", &device_error, "Read and clear kernel error flags (synchronises)");
}
