// Allocation-free variant of the ring-attention block step.
//
// fl_flash2_fwd_block keeps the running attention state of a query block (the
// normalised fp32 output and its log-sum-exp) in buffers the caller
// allocates. Some callers cannot allocate device memory when they call us:
// host runtimes that own all device memory and hand out nothing after
// start-up (an inference server's memory planner, an engine with a fixed
// device-memory budget), or code on a latency-critical path where an
// allocation may stall or fail. fl_flash2_fwd_block_noalloc serves them: the
// running state lives in a fixed array compiled into this library, so the
// caller passes only q, k, v and the fp16 output.

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/flashlite_b200.h"
#include "fl_internal.h"

namespace {

// Largest running state the array holds: B*H*Nq query rows.
constexpr int64_t kNoAllocMaxRows = 65536;
constexpr int64_t kHeadDim = 64;
// Layout: [rows][64] fp32 output, then [rows] fp32 log-sum-exp.
constexpr size_t kScratchFloats = kNoAllocMaxRows * kHeadDim + kNoAllocMaxRows;

}  // namespace

// 17,039,360 bytes (16.25 MiB) of device memory, held by every GPU that loads
// this library until the process exits. In host code this name is only a
// stand-in for the symbol, never a device address: the address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

namespace {

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int fail(int status, const std::string& msg) {
  fl::set_last_error(msg);
  return status;
}

// Device address of the scratch array on the current device, looked up once
// per device (the first call on each device) with that device current.
int scratch_for_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0) return fail(FL_ERR_NO_DEVICE, "no CUDA device");
  if (dev >= kMaxDevices) return fail(FL_ERR_UNSUPPORTED, "device index too large");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FL_ERR_CUDA, std::string("scratch address lookup: ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return FL_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int fl_flash2_fwd_block_noalloc(const void* q, const void* k, const void* v, void* o,
                                           int64_t BH, int64_t Nq, int64_t Nk, int64_t D,
                                           int64_t q_offset, int64_t kv_offset, float sm_scale,
                                           int is_causal, int first, int last, void* stream) {
  if (!q || !k || !v || (last && !o)) return fail(FL_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (BH < 0 || Nq < 0 || Nk < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative size");
  if (D != kHeadDim) return fail(FL_ERR_UNSUPPORTED, "block kernel requires head_dim == 64");
  if (q_offset < 0 || kv_offset < 0) return fail(FL_ERR_INVALID_ARGUMENT, "negative offset");
  if (Nk > (1LL << 30)) return fail(FL_ERR_INVALID_ARGUMENT, "dimension too large");
  if (BH > 0 && Nq > kNoAllocMaxRows / BH)
    return fail(FL_ERR_UNSUPPORTED,
                "B*H*Nq = " + std::to_string(BH * Nq) +
                    " rows exceeds the 65536-row state of the allocation-free entry point; "
                    "use fl_flash2_fwd_block with caller-owned buffers");
  if (BH == 0 || Nq == 0) return FL_OK;
  if (Nk == 0) return fail(FL_ERR_INVALID_ARGUMENT, "empty key block");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (last && (reinterpret_cast<uintptr_t>(o) & 3u)))
    return fail(FL_ERR_MISALIGNED, "q, k, v must be 16-byte and o 4-byte aligned");
  int major = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return fail(FL_ERR_NO_DEVICE, "no CUDA device");
  if (major != 10) return fail(FL_ERR_NO_DEVICE, "flashlite_b200 kernels are built for sm_100a (B200)");
  if (!fl::prepare_current_device()) return fail(FL_ERR_CUDA, "device initialisation failed");
  float* scratch = nullptr;
  int st = scratch_for_current_device(&scratch);
  if (st != FL_OK) return st;
  float* o_acc = scratch;                                // [BH, Nq, 64]
  float* lse = scratch + kNoAllocMaxRows * kHeadDim;     // [BH, Nq]
  double scale = sm_scale;
  if (scale == 0.0) scale = 1.0f / std::sqrt(static_cast<float>(D));
  const float scale_log2 = static_cast<float>(scale * 1.44269504088896340736);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = fl::launch_flash2(q, k, v, nullptr, o_acc, lse, 1, BH, Nq, Nk, q_offset,
                                    kv_offset, scale_log2, is_causal != 0, true, first != 0, false, s);
  if (e != cudaSuccess) return fail(FL_ERR_CUDA, std::string("block launch: ") + cudaGetErrorString(e));
  if (last) {
    e = fl::launch_ring_finalize(o_acc, o, BH * Nq * kHeadDim, s);
    if (e != cudaSuccess)
      return fail(FL_ERR_CUDA, std::string("finalize launch: ") + cudaGetErrorString(e));
  }
  return FL_OK;
}
