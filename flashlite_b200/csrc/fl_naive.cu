// Naive attention forward: the simple, obviously-correct CUDA-core baseline.
//
// Same contract as the reference naive kernel (thebigblender/FlashLite
// csrc/kernel_naive.cu:125-237): one CTA per query row, fp32 dot products
// scaled by sm_scale, natural-base softmax, fp32 P·V, any head_dim. Unlike the
// reference it keeps at most kChunk scores in shared memory and combines
// chunks with an online-softmax rescale, so any sequence length launches
// (the reference needs 4·N bytes of dynamic shared memory and stops
// launching near N = 12k), and it walks query rows with a grid-stride loop
// so B·H is not limited by gridDim.y/z. For D % 8 == 0 on 16-byte aligned
// tensors a second form of the same per-row algorithm reads each key row
// with 16-byte loads shared by eight lanes (whole rows per warp load instead
// of 2-byte loads from 32 different rows) and spreads P·V over all threads;
// other head dims take the scalar form.
//
// Also hosts the ring-attention finalisation (fp32 -> fp16 cast).

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

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

// Vectorised form of the same per-row algorithm, for D % 8 == 0 and 16-byte
// aligned tensors. Scores: eight lanes share one key row, each lane loads
// 16 bytes (8 halves) per step so a warp reads four whole rows per load, and
// the partial dot products are summed with three shuffles. The q row sits in
// registers, QC chunks of 8 per lane (QC = ceil(D / 64) rounded up to a power
// of two). P·V: threads own half2 column pairs; when the row has fewer than
// 128 pairs, G = 128 / pairs key groups run interleaved key ranges and their
// partial sums meet in shared memory.
// two packed fp16 values (low half first) as floats
__device__ __forceinline__ float2 halves_to_float2(uint32_t u) {
  return make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(u & 0xffffu))),
                     __half2float(__ushort_as_half(static_cast<unsigned short>(u >> 16))));
}

template <int QC>
__global__ void __launch_bounds__(kNaiveThreads) naive_attention_vec_kernel(
    const __half* __restrict__ Q, const __half* __restrict__ K, const __half* __restrict__ V,
    __half* __restrict__ O, long long rows_total, int N, int D, float sm_scale, int causal) {
  extern __shared__ float sm[];
  float* acc = sm;      // D floats
  float* sc = sm + D;   // kChunk scores
  __shared__ float scratch[kNaiveThreads / 32];
  __shared__ float red[2 * kNaiveThreads];  // G * D <= 2 * 128 partial sums

  const int lane = threadIdx.x & 31;
  const int sub = lane & 7;                // lane within the 8-lane key group
  const int kgrp = threadIdx.x >> 3;       // 16 key groups per CTA
  const int D8 = D >> 3;                   // 16-byte chunks per row
  const int CP = D >> 1;                   // half2 column pairs per row
  const int G = CP >= kNaiveThreads ? 1 : kNaiveThreads / CP;
  const int pv_g = threadIdx.x / CP;       // key group of this thread in P·V (G > 1)
  const int pv_cp = threadIdx.x % CP;

  for (long long rid = blockIdx.x; rid < rows_total; rid += gridDim.x) {
    const long long bh = rid / N;
    const int i = static_cast<int>(rid % N);
    const __half* kb = K + bh * static_cast<long long>(N) * D;
    const __half* vb = V + bh * static_cast<long long>(N) * D;
    const uint4* qr = reinterpret_cast<const uint4*>(Q + rid * D);

    float qf[QC][8];
#pragma unroll
    for (int c = 0; c < QC; ++c) {
      const int ch = sub + 8 * c;
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (ch < D8) raw = __ldg(qr + ch);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = halves_to_float2(w[e]);
        qf[c][2 * e] = f.x;
        qf[c][2 * e + 1] = f.y;
      }
    }
    for (int d = threadIdx.x; d < D; d += kNaiveThreads) acc[d] = 0.0f;
    __syncthreads();

    const int kv_len = causal ? i + 1 : N;
    float m = -INFINITY, l = 0.0f;
    for (int c0 = 0; c0 < kv_len; c0 += kChunk) {
      const int cn = min(kChunk, kv_len - c0);
      float tmax = -INFINITY;
      // the loop bound is the same for every thread: shuffles stay uniform
      for (int jb = 0; jb < cn; jb += kNaiveThreads / 8) {
        const int j = jb + kgrp;
        float dot = 0.0f;
        if (j < cn) {
          const uint4* kr = reinterpret_cast<const uint4*>(kb + static_cast<long long>(c0 + j) * D);
#pragma unroll
          for (int c = 0; c < QC; ++c) {
            const int ch = sub + 8 * c;
            if (ch < D8) {
              const uint4 raw = __ldg(kr + ch);
              const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = halves_to_float2(w[e]);
                dot = fmaf(qf[c][2 * e], f.x, dot);
                dot = fmaf(qf[c][2 * e + 1], f.y, dot);
              }
            }
          }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        if (sub == 0 && j < cn) {
          const float s = dot * sm_scale;
          sc[j] = s;
          tmax = fmaxf(tmax, s);
        }
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

      const __half2* vc = reinterpret_cast<const __half2*>(vb + static_cast<long long>(c0) * D);
      if (G > 1) {
        if (pv_g < G) {
          float2 a = make_float2(0.0f, 0.0f), b = make_float2(0.0f, 0.0f);
          int j = pv_g;
          for (; j + G < cn; j += 2 * G) {
            const float2 v0 = __half22float2(vc[static_cast<long long>(j) * CP + pv_cp]);
            const float2 v1 = __half22float2(vc[static_cast<long long>(j + G) * CP + pv_cp]);
            const float p0 = sc[j], p1 = sc[j + G];
            a.x = fmaf(p0, v0.x, a.x);
            a.y = fmaf(p0, v0.y, a.y);
            b.x = fmaf(p1, v1.x, b.x);
            b.y = fmaf(p1, v1.y, b.y);
          }
          if (j < cn) {
            const float2 v0 = __half22float2(vc[static_cast<long long>(j) * CP + pv_cp]);
            a.x = fmaf(sc[j], v0.x, a.x);
            a.y = fmaf(sc[j], v0.y, a.y);
          }
          red[pv_g * D + 2 * pv_cp] = a.x + b.x;
          red[pv_g * D + 2 * pv_cp + 1] = a.y + b.y;
        }
        __syncthreads();
        for (int d = threadIdx.x; d < D; d += kNaiveThreads) {
          float s = acc[d] * alpha;
          for (int g = 0; g < G; ++g) s += red[g * D + d];
          acc[d] = s;
        }
      } else {
        for (int cp = threadIdx.x; cp < CP; cp += kNaiveThreads) {
          float2 a = make_float2(0.0f, 0.0f), b = make_float2(0.0f, 0.0f);
          int j = 0;
          for (; j + 1 < cn; j += 2) {
            const float2 v0 = __half22float2(vc[static_cast<long long>(j) * CP + cp]);
            const float2 v1 = __half22float2(vc[static_cast<long long>(j + 1) * CP + cp]);
            const float p0 = sc[j], p1 = sc[j + 1];
            a.x = fmaf(p0, v0.x, a.x);
            a.y = fmaf(p0, v0.y, a.y);
            b.x = fmaf(p1, v1.x, b.x);
            b.y = fmaf(p1, v1.y, b.y);
          }
          if (j < cn) {
            const float2 v0 = __half22float2(vc[static_cast<long long>(j) * CP + cp]);
            a.x = fmaf(sc[j], v0.x, a.x);
            a.y = fmaf(sc[j], v0.y, a.y);
          }
          acc[2 * cp] = acc[2 * cp] * alpha + (a.x + b.x);
          acc[2 * cp + 1] = acc[2 * cp + 1] * alpha + (a.y + b.y);
        }
      }
      m = m_new;
      __syncthreads();  // sc, red and acc settled before the next chunk
    }
    const float inv_l = (l > 0.0f) ? 1.0f / l : 0.0f;
    __half2* orow = reinterpret_cast<__half2*>(O + rid * D);
    for (int cp = threadIdx.x; cp < CP; cp += kNaiveThreads)
      orow[cp] = __floats2half2_rn(acc[2 * cp] * inv_l, acc[2 * cp + 1] * inv_l);
    __syncthreads();  // acc reused by the next row
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
  const long long grid = rows < 148LL * 64 ? rows : 148LL * 64;
  const __half* qh = static_cast<const __half*>(q);
  const __half* kh = static_cast<const __half*>(k);
  const __half* vh = static_cast<const __half*>(v);
  __half* oh = static_cast<__half*>(o);
  const int n = static_cast<int>(N), d = static_cast<int>(D);
  const int causal_i = causal ? 1 : 0;
  const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15u) == 0;
  if (D % 8 == 0 && aligned) {
    // D <= 1024 (checked by the caller) keeps this under the 48 KB default.
    const size_t smem = (static_cast<size_t>(D) + kChunk) * sizeof(float);
    const unsigned g = static_cast<unsigned>(grid);
    const int qc = static_cast<int>((D + 63) / 64);
    if (qc <= 1)
      naive_attention_vec_kernel<1><<<g, kNaiveThreads, smem, stream>>>(qh, kh, vh, oh, rows, n, d, sm_scale, causal_i);
    else if (qc <= 2)
      naive_attention_vec_kernel<2><<<g, kNaiveThreads, smem, stream>>>(qh, kh, vh, oh, rows, n, d, sm_scale, causal_i);
    else if (qc <= 4)
      naive_attention_vec_kernel<4><<<g, kNaiveThreads, smem, stream>>>(qh, kh, vh, oh, rows, n, d, sm_scale, causal_i);
    else if (qc <= 8)
      naive_attention_vec_kernel<8><<<g, kNaiveThreads, smem, stream>>>(qh, kh, vh, oh, rows, n, d, sm_scale, causal_i);
    else
      naive_attention_vec_kernel<16><<<g, kNaiveThreads, smem, stream>>>(qh, kh, vh, oh, rows, n, d, sm_scale, causal_i);
    return cudaGetLastError();
  }
  // D <= 1024 (checked by the caller) keeps this under the 48 KB default.
  const size_t smem = (2 * static_cast<size_t>(D) + kChunk) * sizeof(float);
  naive_attention_kernel<<<static_cast<unsigned>(grid), kNaiveThreads, smem, stream>>>(
      qh, kh, vh, oh, rows, n, d, sm_scale, causal_i);
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
