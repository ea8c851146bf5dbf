// Internal (host-side) declarations shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <string>

namespace fl {

// Per-thread text of the last error; returned by fl_last_error().
void set_last_error(const std::string& msg);
const char* last_error();

// Device-side error word of the current device (address in device memory).
unsigned int* device_error_word();

// Raises `kern`'s dynamic shared-memory limit to `bytes` on the current
// device, once per device and kernel. Thread-safe: `done` (one per kernel
// instantiation, static storage) records the devices already configured; two
// threads may both configure a device the first time, which is harmless
// (cudaFuncSetAttribute is idempotent). Devices past kMaxFlagDevices are
// configured on every call.
constexpr int kMaxFlagDevices = 64;
template <typename Kernel>
cudaError_t ensure_smem_limit(Kernel kern, int bytes, std::atomic<bool> (&done)[kMaxFlagDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < kMaxFlagDevices;
  if (tracked && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && tracked) done[dev].store(true, std::memory_order_release);
  return e;
}

// Number of SMs of the current device (cached per device).
int sm_count();

// Caches the current device's attributes and error-word address (what the
// C-ABI entry points do before their first launch); false on failure.
bool prepare_current_device();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link dependency); nullptr when unavailable.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn get_encode_fn();

// fp16 tensor map {D, rows, H, B} over [B,H,rows,D] (bnhd = false) or
// [B,rows,H,D] (bnhd = true), box {64, box_rows, 1, 1}, 128-byte swizzle.
bool encode_rows_map(CUtensorMap* tm, const void* base, int64_t rows, int64_t H, int64_t B,
                     bool bnhd, int D, int box_rows);

// Launchers. All sizes validated by the caller; return 0 or a cudaError_t.
// q/k/v/o are [B,H,N,D] fp16, or [B,N,H,D] with bnhd (non-merge only);
// head_dim D is 64 or 128.
cudaError_t launch_flash2(const void* q, const void* k, const void* v, void* o_f16, float* o_acc,
                          float* lse, int64_t B, int64_t H, int64_t Nq, int64_t Nk,
                          int64_t q_offset, int64_t kv_offset, float scale_log2, bool causal,
                          bool merge, bool first, bool bnhd, cudaStream_t stream,
                          int head_dim = 64);

// FA2 backward (head_dim 64, [B,H,N,64] or with bnhd [B,N,H,64] fp16): dq, dk, dv from q, k, v, the
// forward output o, its gradient dout and the forward's natural-log LSE
// [B,H,N] fp32. workspace: flash2_bwd_workspace_bytes(B*H, N) bytes.
size_t flash2_bwd_workspace_bytes(int64_t BH, int64_t N);
cudaError_t launch_flash2_bwd(const void* q, const void* k, const void* v, const void* o,
                              const void* dout, const float* lse, void* dq, void* dk, void* dv,
                              void* workspace, int64_t B, int64_t H, int64_t N, float sm_scale,
                              bool causal, bool bnhd, cudaStream_t stream, const char** where);

cudaError_t launch_naive(const void* q, const void* k, const void* v, void* o, int64_t BH,
                         int64_t N, int64_t D, float sm_scale, bool causal, cudaStream_t stream);

cudaError_t launch_ring_finalize(const float* o_acc, void* o, int64_t n, cudaStream_t stream);

}  // namespace fl
