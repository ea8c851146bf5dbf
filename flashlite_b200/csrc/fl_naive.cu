// Naive attention forward: the simple, obviously-correct CUDA-core baseline.
//
// Same contract as the reference naive kernel (thebigblender/FlashLite
// csrc/kernel_naive.cu:125-237): one CTA per query row, fp32 dot products
// scaled by sm_scale, natural-base softmax, fp32 P·V, any head_dim. Unlike the
// reference it keeps at most kChunk scores in shared memory and combines
// chunks with an online-softmax rescale, so any sequence length launches
// (the reference needs 4·N bytes of dynamic shared memory and stops
// launching near N = 12k), and it walks query rows with a grid-stride loop
// so B·H is not limited by gridDim.y/z.
//
// Also hosts the ring-attention finalisation (fp32 -> fp16 cast).

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "fl_internal.h"

namespace fl {
namespace {

constexpr int kNaiveThreads = 128;
constexpr int kChunk = 2048;  // scores held in shared memory per pass

__device__ __forceinline__ float block_reduce(float v, float* scratch, bool is_max) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();  // scratch may still be read from the previous reduction
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  float r = scratch[0];
  for (int w = 1; w < kNaiveThreads / 32; ++w) r = is_max ? fmaxf(r, scratch[w]) : r + scratch[w];
  return r;
}

// dynamic shared memory: q row (D floats) | acc (D floats) | scores (kChunk)
__global__ void __launch_bounds__(kNaiveThreads) naive_attention_kernel(
    const __half* __restrict__ Q, const __half* __restrict__ K, const __half* __restrict__ V,
    __half* __restrict__ O, long long rows_total, int N, int D, float sm_scale, int causal) {
  extern __shared__ float sm[];
  float* q_s = sm;
  float* acc = sm + D;
  float* sc = sm + 2 * D;
  __shared__ float scratch[kNaiveThreads / 32];

  for (long long rid = blockIdx.x; rid < rows_total; rid += gridDim.x) {
    const long long bh = rid / N;
    const int i = static_cast<int>(rid % N);
    const __half* kb = K + bh * static_cast<long long>(N) * D;
    const __half* vb = V + bh * static_cast<long long>(N) * D;
    const __half* qr = Q + rid * D;

    for (int d = threadIdx.x; d < D; d += kNaiveThreads) {
      q_s[d] = __half2float(qr[d]);
      acc[d] = 0.0f;
    }
    __syncthreads();

    const int kv_len = causal ? i + 1 : N;
    float m = -INFINITY, l = 0.0f;
    for (int c0 = 0; c0 < kv_len; c0 += kChunk) {
      const int cn = min(kChunk, kv_len - c0);
      float tmax = -INFINITY;
      for (int j = threadIdx.x; j < cn; j += kNaiveThreads) {
        const __half* kr = kb + static_cast<long long>(c0 + j) * D;
        float dot = 0.0f;
        for (int d = 0; d < D; ++d) dot = fmaf(q_s[d], __half2float(kr[d]), dot);
        const float s = dot * sm_scale;
        sc[j] = s;
        tmax = fmaxf(tmax, s);
      }
      const float m_new = fmaxf(m, block_reduce(tmax, scratch, true));
      const float alpha = (m == -INFINITY) ? 0.0f : expf(m - m_new);
      float tsum = 0.0f;
      for (int j = threadIdx.x; j < cn; j += kNaiveThreads) {
        const float pj = expf(sc[j] - m_new);
        sc[j] = pj;
        tsum += pj;
      }
      l = l * alpha + block_reduce(tsum, scratch, false);
      __syncthreads();  // all p_j visible
      for (int d = threadIdx.x; d < D; d += kNaiveThreads) {
        float a = acc[d] * alpha;
        const __half* vc = vb + static_cast<long long>(c0) * D + d;
        for (int j = 0; j < cn; ++j) a = fmaf(sc[j], __half2float(vc[static_cast<long long>(j) * D]), a);
        acc[d] = a;
      }
      m = m_new;
      __syncthreads();  // sc reused by the next chunk
    }
    const float inv_l = (l > 0.0f) ? 1.0f / l : 0.0f;
    __half* orow = O + rid * D;
    for (int d = threadIdx.x; d < D; d += kNaiveThreads) orow[d] = __float2half_rn(acc[d] * inv_l);
    __syncthreads();  // q_s/acc reused by the next row
  }
}

__global__ void f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, long long n) {
  long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 4;
  for (; i < n; i += stride) {
    if (i + 3 < n) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
      *reinterpret_cast<__half2*>(dst + i) = a;
      *reinterpret_cast<__half2*>(dst + i + 2) = b;
    } else {
      for (long long e = i; e < n; ++e) dst[e] = __float2half_rn(src[e]);
    }
  }
}

}  // namespace

cudaError_t launch_naive(const void* q, const void* k, const void* v, void* o, int64_t BH,
                         int64_t N, int64_t D, float sm_scale, bool causal, cudaStream_t stream) {
  const long long rows = static_cast<long long>(BH) * N;
  // D <= 1024 (checked by the caller) keeps this under the 48 KB default.
  const size_t smem = (2 * static_cast<size_t>(D) + kChunk) * sizeof(float);
  const long long grid = rows < 148LL * 64 ? rows : 148LL * 64;
  naive_attention_kernel<<<static_cast<unsigned>(grid), kNaiveThreads, smem, stream>>>(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v),
      static_cast<__half*>(o), rows, static_cast<int>(N), static_cast<int>(D), sm_scale,
      causal ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_ring_finalize(const float* o_acc, void* o, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n / 4 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  f32_to_f16_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(o_acc, static_cast<__half*>(o), n);
  return cudaGetLastError();
}

}  // namespace fl
