// C-ABI entry points of libflashlite_b200 (declared in include/flashlite_b200.h).
//
// Validation mirrors the reference host launchers
// (thebigblender/FlashLite csrc/kernel_flash2.cu:741-771 and
// csrc/kernel_naive.cu:252-280) for everything that can be checked on raw
// pointers and sizes; dtype/contiguity/device checks of torch tensors live in
// the torch binding (flash_attn.cpp). No entry point allocates device memory.

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/flashlite_b200.h"
#include "fl_internal.h"

namespace fl {

namespace {
thread_local std::string g_last_error;

// Device error word: kernels OR bit flags into it when they give up a wait.
__device__ unsigned int g_device_error = 0;

constexpr int kMaxDevices = 64;
unsigned int* g_err_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
int g_cc_major[kMaxDevices] = {};
std::mutex g_dev_mu;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

bool init_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return false;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_err_ptr[dev]) return true;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return false;
  int sms = 0, major = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  g_sm_count[dev] = sms;
  g_cc_major[dev] = major;
  g_err_ptr[dev] = static_cast<unsigned int*>(p);
  return true;
}
}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

unsigned int* device_error_word() {
  const int dev = current_device();
  return (dev >= 0 && dev < kMaxDevices) ? g_err_ptr[dev] : nullptr;
}

bool prepare_current_device() {
  const int dev = current_device();
  // binds the primary context to this thread (see check_device)
  if (dev < 0 || cudaSetDevice(dev) != cudaSuccess) return false;
  return init_device(dev);
}

int sm_count() {
  const int dev = current_device();
  return (dev >= 0 && dev < kMaxDevices && g_sm_count[dev] > 0) ? g_sm_count[dev] : 148;
}

}  // namespace fl

namespace {

int fail(int status, const std::string& msg) {
  fl::set_last_error(msg);
  return status;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(FL_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

// Checks shared by the attention entry points; returns FL_OK or an error.
int check_common(const void* q, const void* k, const void* v, const void* o, int64_t B, int64_t H,
                 int64_t N, int64_t D) {
  if (!q || !k || !v || !o) return fail(FL_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (B < 0 || H < 0 || N < 0 || D <= 0)
    return fail(FL_ERR_INVALID_ARGUMENT, "Tensors must be 4D [B, H, N, D] with non-negative sizes");
  // every element offset must fit comfortably in 64-bit and N in 32-bit
  if (N > (1LL << 30) || B > (1LL << 30) || H > (1LL << 30))
    return fail(FL_ERR_INVALID_ARGUMENT, "dimension too large");
  const long double elems = static_cast<long double>(B) * H * N * D;
  if (elems > static_cast<long double>(1LL << 46))
    return fail(FL_ERR_INVALID_ARGUMENT, "tensor too large");
  return FL_OK;
}

int check_device() {
  const int dev = fl::current_device();
  if (dev < 0) return fail(FL_ERR_NO_DEVICE, "no CUDA device");
  // Bind the device's primary context to this thread: tensor maps are encoded
  // through the driver API before the first runtime launch, and a thread
  // that has only queried the device (an autograd worker, say) has no
  // current context yet.
  if (cudaSetDevice(dev) != cudaSuccess) return fail(FL_ERR_NO_DEVICE, "cannot bind the CUDA device");
  if (!fl::init_device(dev)) return fail(FL_ERR_CUDA, "device initialisation failed");
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return fail(FL_ERR_NO_DEVICE, "flashlite_b200 kernels are built for sm_100a (B200)");
  return FL_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

const char* fl_version(void) { return "0.1.0"; }

const char* fl_status_str(int status) {
  switch (status) {
    case FL_OK: return "ok";
    case FL_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FL_ERR_UNSUPPORTED: return "unsupported configuration";
    case FL_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case FL_ERR_CUDA: return "CUDA error";
    case FL_ERR_NO_DEVICE: return "no sm_100 device";
    case FL_ERR_DEVICE_TIMEOUT: return "a kernel wait timed out";
    default: return "unknown status";
  }
}

const char* fl_last_error(void) { return fl::last_error(); }

int fl_flash2_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
                  int64_t N, int64_t D, float sm_scale, int is_causal, void* stream) {
  int st = check_common(q, k, v, o, B, H, N, D);
  if (st != FL_OK) return st;
  // csrc/kernel_flash2.cu:756-757
  if (D != 64) return fail(FL_ERR_UNSUPPORTED, "FlashLite WMMA kernel currently requires head_dim == 64");
  if (B == 0 || H == 0 || N == 0) return FL_OK;  // empty output, nothing to compute
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(FL_ERR_MISALIGNED, "q, k, v and out must be 16-byte aligned");
  if ((st = check_device()) != FL_OK) return st;
  // csrc/kernel_flash2.cu:769-772
  double scale = sm_scale;
  if (scale == 0.0) scale = 1.0f / std::sqrt(static_cast<float>(D));
  const float scale_log2 = static_cast<float>(scale * 1.44269504088896340736);
  cudaError_t e = fl::launch_flash2(q, k, v, o, nullptr, nullptr, B, H, N, N, 0, 0, scale_log2,
                                    is_causal != 0, false, false, false,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "flash2 launch");
  return FL_OK;
}

int fl_flash2_fwd_ex(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                     int64_t H, int64_t Nq, int64_t Nk, int64_t D, int64_t q_offset,
                     int64_t kv_offset, float sm_scale, int is_causal, int layout, void* stream) {
  if (!q || !k || !v || !o) return fail(FL_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (layout != FL_LAYOUT_BHND && layout != FL_LAYOUT_BNHD)
    return fail(FL_ERR_INVALID_ARGUMENT, "unknown layout");
  if (B < 0 || H < 0 || Nq < 0 || Nk < 0 || D < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative size");
  if (Nq > (1LL << 30) || Nk > (1LL << 30) || B * H > (1LL << 30))
    return fail(FL_ERR_INVALID_ARGUMENT, "dimension too large");
  if (q_offset < 0 || kv_offset < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative offset");
  if (D != 64 && D != 128) return fail(FL_ERR_UNSUPPORTED, "forward_flash2_ex requires head_dim 64 or 128");
  if (B == 0 || H == 0 || Nq == 0) return FL_OK;
  if (Nk == 0) return fail(FL_ERR_INVALID_ARGUMENT, "empty key sequence");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(FL_ERR_MISALIGNED, "q, k, v and out must be 16-byte aligned");
  int st = check_device();
  if (st != FL_OK) return st;
  double scale = sm_scale;
  if (scale == 0.0) scale = 1.0f / std::sqrt(static_cast<float>(D));
  const float scale_log2 = static_cast<float>(scale * 1.44269504088896340736);
  cudaError_t e = fl::launch_flash2(q, k, v, o, nullptr, lse, B, H, Nq, Nk, q_offset, kv_offset,
                                    scale_log2, is_causal != 0, false, false,
                                    layout == FL_LAYOUT_BNHD, static_cast<cudaStream_t>(stream),
                                    static_cast<int>(D));
  if (e != cudaSuccess) return cuda_fail(e, "flash2 launch");
  return FL_OK;
}

int fl_naive_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
                 int64_t N, int64_t D, float sm_scale, int is_causal, void* stream) {
  int st = check_common(q, k, v, o, B, H, N, D);
  if (st != FL_OK) return st;
  if (D > 1024) return fail(FL_ERR_UNSUPPORTED, "naive kernel supports head_dim <= 1024");
  if (B == 0 || H == 0 || N == 0) return FL_OK;
  if ((st = check_device()) != FL_OK) return st;
  // csrc/kernel_naive.cu:278-280
  double scale = sm_scale;
  if (scale == 0.0) scale = 1.0f / std::sqrt(static_cast<float>(D));
  cudaError_t e = fl::launch_naive(q, k, v, o, B * H, N, D, static_cast<float>(scale),
                                   is_causal != 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "naive launch");
  return FL_OK;
}

int fl_flash2_fwd_block(const void* q, const void* k, const void* v, float* o_acc, float* lse,
                        int64_t BH, int64_t Nq, int64_t Nk, int64_t D, int64_t q_offset,
                        int64_t kv_offset, float sm_scale, int is_causal, int first,
                        void* stream) {
  if (!q || !k || !v || !o_acc || !lse) return fail(FL_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (BH < 0 || Nq < 0 || Nk < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative size");
  if (D != 64 && D != 128) return fail(FL_ERR_UNSUPPORTED, "block kernel requires head_dim 64 or 128");
  if (Nq > (1LL << 30) || Nk > (1LL << 30) || BH > (1LL << 30))
    return fail(FL_ERR_INVALID_ARGUMENT, "dimension too large");
  if (q_offset < 0 || kv_offset < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative offset");
  if (BH == 0 || Nq == 0) return FL_OK;
  if (Nk == 0) return fail(FL_ERR_INVALID_ARGUMENT, "empty key block");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o_acc))
    return fail(FL_ERR_MISALIGNED, "q, k, v and o_acc must be 16-byte aligned");
  int st = check_device();
  if (st != FL_OK) return st;
  double scale = sm_scale;
  if (scale == 0.0) scale = 1.0f / std::sqrt(static_cast<float>(D));
  const float scale_log2 = static_cast<float>(scale * 1.44269504088896340736);
  cudaError_t e = fl::launch_flash2(q, k, v, nullptr, o_acc, lse, 1, BH, Nq, Nk, q_offset,
                                    kv_offset, scale_log2, is_causal != 0, true, first != 0, false,
                                    static_cast<cudaStream_t>(stream), static_cast<int>(D));
  if (e != cudaSuccess) return cuda_fail(e, "flash2 block launch");
  return FL_OK;
}

int fl_ring_finalize(const float* o_acc, void* o, int64_t n_elems, void* stream) {
  if (n_elems < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative size");
  if (n_elems == 0) return FL_OK;
  if (!o_acc || !o) return fail(FL_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned16(o_acc) || (reinterpret_cast<uintptr_t>(o) & 3u))
    return fail(FL_ERR_MISALIGNED, "o_acc must be 16-byte and o 4-byte aligned");
  int st = check_device();
  if (st != FL_OK) return st;
  cudaError_t e = fl::launch_ring_finalize(o_acc, o, n_elems, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "finalize launch");
  return FL_OK;
}

size_t fl_flash2_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D) {
  if (B <= 0 || H <= 0 || N <= 0 || D != 64 || N > (1LL << 30) || B * H > (1LL << 30)) return 0;
  return fl::flash2_bwd_workspace_bytes(B * H, N);
}

int fl_flash2_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, void* workspace,
                  size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D,
                  float sm_scale, int is_causal, int layout, void* stream) {
  int st = check_common(q, k, v, o, B, H, N, D);
  if (st != FL_OK) return st;
  if (!dout || !lse || !dq || !dk || !dv) return fail(FL_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (layout != FL_LAYOUT_BHND && layout != FL_LAYOUT_BNHD)
    return fail(FL_ERR_INVALID_ARGUMENT, "unknown layout");
  if (D != 64) return fail(FL_ERR_UNSUPPORTED, "backward_flash2 requires head_dim == 64");
  if (B == 0 || H == 0 || N == 0) return FL_OK;
  if (B * H > (1LL << 30)) return fail(FL_ERR_INVALID_ARGUMENT, "dimension too large");
  const size_t need = fl::flash2_bwd_workspace_bytes(B * H, N);
  if (!workspace || workspace_bytes < need)
    return fail(FL_ERR_INVALID_ARGUMENT,
                "workspace too small: " + std::to_string(need) + " bytes needed (fl_flash2_bwd_workspace_size)");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dout) ||
      !aligned16(dk) || !aligned16(dv) || !aligned16(workspace) || (reinterpret_cast<uintptr_t>(dq) & 3u) ||
      (reinterpret_cast<uintptr_t>(lse) & 3u))
    return fail(FL_ERR_MISALIGNED, "q, k, v, out, dout, dk, dv and workspace must be 16-byte aligned");
  st = check_device();
  if (st != FL_OK) return st;
  double scale = sm_scale;
  if (scale == 0.0) scale = 1.0f / std::sqrt(static_cast<float>(D));
  const char* where = "flash2 backward";
  cudaError_t e = fl::launch_flash2_bwd(q, k, v, o, dout, lse, dq, dk, dv, workspace, B, H, N,
                                        static_cast<float>(scale), is_causal != 0,
                                        layout == FL_LAYOUT_BNHD, static_cast<cudaStream_t>(stream), &where);
  if (e != cudaSuccess) return cuda_fail(e, (std::string("flash2 backward: ") + where).c_str());
  return FL_OK;
}

int fl_device_error(void* stream, uint32_t* flags) {
  int st = check_device();
  if (st != FL_OK) return st;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  unsigned int word = 0;
  e = cudaMemcpyFromSymbol(&word, fl::g_device_error, sizeof(word));
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  if (word) {
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(fl::g_device_error, &zero, sizeof(zero));
  }
  if (flags) *flags = word;
  return word ? fail(FL_ERR_DEVICE_TIMEOUT, "a kernel gave up a bounded wait") : FL_OK;
}

}  // extern "C"
