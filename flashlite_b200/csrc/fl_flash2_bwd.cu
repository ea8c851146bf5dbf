// FlashAttention-2 backward for B200 (sm_100a), head_dim 64, fp16 in/out.
//
// No reference counterpart: thebigblender/FlashLite is forward-only. The
// forward's log-sum-exp output (fl_flash2_fwd_ex) is what this consumes.
// Mathematics (per (b,h) slice, S = scale * Q K^T, P = exp(S - LSE) by row):
//   dV = P^T dO,  dP = dO V^T,  Delta = rowsum(dO * O),
//   dS = P * (dP - Delta),  dQ = scale * dS K,  dK = scale * dS^T Q.
//
// Design:
//  * one CTA per (slice, 128-key tile): K and V stay in shared memory while
//    the CTA streams every query tile that sees them (causal: from the
//    diagonal tile on) through a 2-deep TMA ring of (Q, dO, LSE, Delta).
//  * everything is computed key-major, so TMEM lanes are the CTA's keys:
//    S^T = K Q^T and dP^T = V dO^T land in TMEM (128 columns each); four
//    gradient warpgroups (one thread per key, each taking 32 of the 128
//    query columns: P needs no row reduction since LSE is known) turn them
//    into P^T and dS^T 16 columns at a time, write both back into columns
//    the same warp has already read (fp16 pairs, operand A of the next MMAs:
//    queries 32c .. 32c + 31 sit at columns 32c .. 32c + 15), and write dS^T
//    to shared memory in the MN-major layout that makes it dS, operand A of
//    dQ = dS K. Four such warps per SM sub-partition hide each other's TMEM
//    and MUFU latency.
//  * the MMA warp then issues dV += P^T dO and dK += dS^T Q (A from TMEM,
//    accumulated over the query tiles in TMEM) and dQ_i = dS K (A and B
//    from shared memory, K read as MN-major B).
//  * a second warpgroup drains dQ_i (one thread per query row): TMEM ->
//    scaled fp32 rows in shared memory -> one TMA reduce-add into an fp32
//    dQ accumulator in global memory (several key tiles add into each query
//    tile); a final pass casts it to fp16.
//  * every mbarrier wait is bounded (see fl_ptx.cuh); on timeout the CTA
//    drains its copies and MMAs, frees TMEM and returns with an error bit.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>

#include "fl_internal.h"
#include "fl_ptx.cuh"

namespace fl {
namespace {

constexpr int kBM = 128;                  // query rows per tile
constexpr int kBK = 128;                  // keys per CTA
constexpr int kD = 64;                    // head dimension
constexpr int kThreads = 768;             // producer/MMA | gradient x 4 | dQ drain
constexpr int kTile = 128 * kD * 2;       // 16 KB: one 128 x 64 fp16 tile
constexpr int kStages = 2;                // (Q, dO, LSE, Delta) ring depth
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S^T then P^T (fp16 pairs in its first 64 columns), dP^T then
// dS^T (likewise), the dV and dK accumulators, dQ of the current query tile.
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 320, kColDQ = 384;

// Shared-memory map (offsets from a 1024-byte aligned base).
constexpr int kSmemK = 0;
constexpr int kSmemV = kSmemK + kTile;
constexpr int kSmemQ = kSmemV + kTile;                 // kStages tiles
constexpr int kSmemDO = kSmemQ + kStages * kTile;      // kStages tiles
constexpr int kSmemDS = kSmemDO + kStages * kTile;     // 2 x dS, 128 x 128 fp16, MN-major
constexpr int kSmemDQ = kSmemDS + 4 * kTile;           // dQ staging, 128 x 64 fp32
constexpr int kSmemVec = kSmemDQ + kBM * kD * 4;       // kStages x (lse2[128], delta[128])
constexpr int kSmemBar = kSmemVec + kStages * 2 * kBM * 4;
// kv_full | q_full, q_empty (x kStages) | s_full, p_full (x 2 query halves) | mm_done |
// dq_free | final
constexpr int kNumBars = 1 + 2 * kStages + 7;
constexpr int kSmemMisc = kSmemBar + kNumBars * 8;     // tmem base, abort flag
constexpr int kSmemAlloc = kSmemMisc + 16 + 1024;
static_assert(kSmemAlloc <= 227 * 1024, "shared memory");

struct BwdParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_do;  // fp16 {64, N, H, B}, box {64, 128}, SW128
  CUtensorMap tm_dq;                    // fp32 {64, N, H, B} dQ accumulator, box {32, 128}, SW128
  const float* lse2;   // [BH, npad] LSE * log2(e), +inf past N
  const float* delta;  // [BH, npad] rowsum(dO * O), 0 past N
  __half* dk;          // [B, H, N, 64] (bnhd: [B, N, H, 64])
  __half* dv;
  unsigned int* err;
  int n, npad, bh, nh, n_tiles;
  int bnhd;            // layout of q, k, v, o, dout, dq, dk, dv
  float scale_log2;    // sm_scale * log2(e)
  float scale;         // sm_scale
};

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int* err) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ bool warp_wait_issuer(uint32_t bar, uint32_t parity,
                                                 volatile int* abort_flag, unsigned int* err) {
  const bool ok = mbar_wait_issuer(bar, parity, abort_flag, err);
  return __all_sync(0xffffffffu, ok);
}

template <bool kCausal>
__global__ void __launch_bounds__(kThreads, 1) flash2_bwd_kernel(const __grid_constant__ BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t s_k = sbase + kSmemK, s_v = sbase + kSmemV;
  const uint32_t s_ds = sbase + kSmemDS, s_dq = sbase + kSmemDQ;
  auto s_q = [&](int st) { return sbase + kSmemQ + st * kTile; };
  auto s_do = [&](int st) { return sbase + kSmemDO + st * kTile; };
  auto s_vec = [&](int st) { return sbase + kSmemVec + st * 2 * kBM * 4; };
  const uint32_t bar0 = sbase + kSmemBar;
  const uint32_t bar_kv = bar0;
  auto bar_qfull = [&](int st) { return bar0 + 8u * (1 + st); };
  auto bar_qempty = [&](int st) { return bar0 + 8u * (1 + kStages + st); };
  const uint32_t bar_x = bar0 + 8u * (1 + 2 * kStages);
  auto bar_s = [&](int h) { return bar_x + 8u * h; };        // S^T, dP^T of query half h in TMEM
  auto bar_p = [&](int h) { return bar_x + 8u * (2 + h); };  // P^T, dS^T of half h written
  const uint32_t bar_mm = bar_x + 32;                       // all MMAs of a query tile done
  const uint32_t bar_dqfree = bar_x + 40;                   // dQ columns read out
  const uint32_t bar_final = bar_x + 48;                    // every MMA of the CTA done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work unit: (key tile jt, slice bh); causal launches the longest first ----
  int jt, bh;
  if (kCausal) {
    jt = blockIdx.x / p.bh;
    bh = blockIdx.x % p.bh;
  } else {
    jt = blockIdx.x % p.n_tiles;
    bh = blockIdx.x / p.n_tiles;
  }
  const int kv_start = jt * kBK;
  const int i0 = kCausal ? jt : 0;  // first query tile that sees these keys
  const int nq = p.n_tiles - i0;    // >= 1
  const int h = bh % p.nh, b = bh / p.nh;

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int st = 0; st < kStages; ++st) {
      mbar_init(bar_qfull(st), 1);
      mbar_init(bar_qempty(st), 1);
    }
    for (int hq = 0; hq < 2; ++hq) {
      mbar_init(bar_s(hq), 1);
      mbar_init(bar_p(hq), 8);  // one arrival per gradient warp of that half
    }
    mbar_init(bar_mm, 1);
    mbar_init(bar_dqfree, 4);  // one arrival per dQ warp
    mbar_init(bar_final, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: set-up above overlaps the preprocess
  // kernel; its Delta / LSE rows (and the cleared dQ accumulator) are read
  // only after this wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ======================= TMA producer =======================
    int issued = 0;
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_do);
      mbar_arrive_expect_tx(bar_kv, 2 * kTile);
      tma_load_4d(s_k, &p.tm_k, bar_kv, 0, kv_start, h, b);
      tma_load_4d(s_v, &p.tm_v, bar_kv, 0, kv_start, h, b);
    }
    __syncwarp();
    for (int it = 0; it < nq; ++it) {
      const int st = it % kStages;
      if (!warp_wait(bar_qempty(st), ((it / kStages) & 1) ^ 1, abort_flag, p.err)) break;
      if (lane == 0) {
        const int qi = i0 + it;
        const long long vec = static_cast<long long>(bh) * p.npad + static_cast<long long>(qi) * kBM;
        mbar_arrive_expect_tx(bar_qfull(st), 2 * kTile + 2 * kBM * 4);
        tma_load_4d(s_q(st), &p.tm_q, bar_qfull(st), 0, qi * kBM, h, b);
        tma_load_4d(s_do(st), &p.tm_do, bar_qfull(st), 0, qi * kBM, h, b);
        bulk_load(s_vec(st), p.lse2 + vec, kBM * 4, bar_qfull(st));
        bulk_load(s_vec(st) + kBM * 4, p.delta + vec, kBM * 4, bar_qfull(st));
      }
      __syncwarp();
      issued = it + 1;
    }
    if (*abort_flag && lane == 0) {
      // let every copy this CTA started land before shared memory is released
      mbar_wait_quiet(bar_kv, 0);
      for (int it = issued > kStages ? issued - kStages : 0; it < issued; ++it)
        mbar_wait_quiet(bar_qfull(it % kStages), (it / kStages) & 1);
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    // Warp-uniform operands, one elected lane issues (as in the forward).
    constexpr uint32_t idesc_s = make_idesc_f16_f32(kBK, kBM / 2, false);      // K-major A, B
    constexpr uint32_t idesc_kv = make_idesc_f16_f32(kBK, kD, true);           // B MN-major
    constexpr uint32_t idesc_dq = make_idesc_f16_f32(kBM, kD, true, true);     // A, B MN-major
    constexpr uint64_t kTileEnc = kTile >> 4;
    const uint32_t tm = __shfl_sync(0xffffffffu, tmem, 0);
    const uint64_t d_k = make_sdesc_sw128(s_k, 16, 1024);        // K as A (K-major)
    const uint64_t d_v = make_sdesc_sw128(s_v, 16, 1024);        // V as A (K-major)
    const uint64_t d_kmn = make_sdesc_sw128(s_k, 8192, 1024);    // K as B of dQ (MN-major)
    const uint64_t d_q0 = make_sdesc_sw128(s_q(0), 16, 1024);    // Q as B of S^T (K-major)
    const uint64_t d_do0 = make_sdesc_sw128(s_do(0), 16, 1024);  // dO as B of dP^T (K-major)
    const uint64_t d_qmn0 = make_sdesc_sw128(s_q(0), 8192, 1024);    // Q as B of dK (MN-major)
    const uint64_t d_domn0 = make_sdesc_sw128(s_do(0), 8192, 1024);  // dO as B of dV (MN-major)
    const uint64_t d_ds = make_sdesc_sw128(s_ds, kTile, 1024);  // dS as A (MN-major; halves 16 KB apart)
    auto commit_to = [&](uint32_t bar) {
      if (elect_one()) umma_commit(bar);
      __syncwarp();
    };
    // S^T, dP^T of query tile `it`, one query half at a time (N = 64; half h's
    // queries are the 8 KB of Q / dO rows 64 h..), so the gradient warps of
    // half 0 start while half 1 is computed
    auto issue_s = [&](int it) {
      const uint64_t so = static_cast<uint64_t>(it % kStages) * kTileEnc;
      if (elect_one()) {
#pragma unroll
        for (int hq = 0; hq < 2; ++hq) {
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            umma_f16_ss(tm + kColS + 64 * hq, d_k + 2 * kk, d_q0 + so + 512 * hq + 2 * kk, idesc_s,
                        kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            umma_f16_ss(tm + kColDP + 64 * hq, d_v + 2 * kk, d_do0 + so + 512 * hq + 2 * kk, idesc_s,
                        kk > 0 ? 1u : 0u);
          umma_commit(bar_s(hq));
        }
      }
      __syncwarp();
    };
    bool ok = warp_wait_issuer(bar_kv, 0, abort_flag, p.err) &&
              warp_wait_issuer(bar_qfull(0), 0, abort_flag, p.err);
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    // Per query tile i: dV, dK of i (as its gradient halves finish), then
    // S^T, dP^T of tile i + 1, then dQ_i, so the gradient warps of tile i + 1
    // work while dQ_i is computed (dS is double-buffered in shared memory).
    for (int it = 0; ok && it < nq; ++it) {
      const int st = it % kStages;
      const uint64_t so = static_cast<uint64_t>(st) * kTileEnc;
      bool done = true;
#pragma unroll
      for (int hq = 0; hq < 2; ++hq) {
        if (!warp_wait_issuer(bar_p(hq), it & 1, abort_flag, p.err)) { done = false; break; }
        tc_fence_after();
        if (elect_one()) {
          // dV += P^T dO and dK += dS^T Q over this half's 64 queries: A from
          // TMEM (16 queries = 8 columns per K step; queries 32c.. at column
          // 32c), B MN-major (16 rows = 2048 B per K step)
#pragma unroll
          for (int kk = 4 * hq; kk < 4 * hq + 4; ++kk)
            umma_f16_ts(tm + kColDV, tm + kColS + 32 * (kk >> 1) + 8 * (kk & 1), d_domn0 + so + 128 * kk,
                        idesc_kv, (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 4 * hq; kk < 4 * hq + 4; ++kk)
            umma_f16_ts(tm + kColDK, tm + kColDP + 32 * (kk >> 1) + 8 * (kk & 1), d_qmn0 + so + 128 * kk,
                        idesc_kv, (it > 0 || kk > 0) ? 1u : 0u);
          // dV, dK of this tile done: Q, dO of the stage and the TMEM columns
          // of P^T, dS^T are free
          if (hq == 1) umma_commit(bar_qempty(st));
        }
        __syncwarp();
      }
      if (!done) break;
      if (it + 1 < nq) {
        if (!warp_wait_issuer(bar_qfull((it + 1) % kStages), ((it + 1) / kStages) & 1, abort_flag, p.err) ||
            !warp_wait_issuer(bar_qempty(st), (it / kStages) & 1, abort_flag, p.err))
          break;
        tc_fence_after();
        issue_s(it + 1);
      }
      // dQ_i = dS_i K (dS buffer i % 2) once the drain warps have read dQ_{i-1}
      if (it > 0 && !warp_wait_issuer(bar_dqfree, (it - 1) & 1, abort_flag, p.err)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t dsb = d_ds + static_cast<uint64_t>(it & 1) * ((4 * kTile / 2) >> 4);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16_ss(tm + kColDQ, dsb + 128 * kk, d_kmn + 128 * kk, idesc_dq, kk > 0 ? 1u : 0u);
        umma_commit(bar_mm);
      }
      __syncwarp();
    }
    // every MMA this thread issued has completed (also the signal for the
    // dK / dV epilogue)
    commit_to(bar_final);
    if (lane == 0) mbar_wait_quiet(bar_final, 0);
    __syncwarp();
  } else if (warp >= 4 && warp < 20) {
    // ======================= gradient warpgroups (one thread per key) =======================
    const int gq = (warp - 4) >> 2;           // query columns 32 gq .. 32 gq + 31
    const int qh = gq >> 1;                   // query half
    const int k = 32 * (warp & 3) + lane;     // key row within the tile = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t tS = tmem + lane_base + kColS;
    const uint32_t tDP = tmem + lane_base + kColDP;
    const float scl = p.scale_log2;
    const float2 scl2 = make_float2(scl, scl);
    // dS^T row k is column k of dS: in the MN-major operand it is row k % 8 of
    // 8-key group k / 8; 16-byte chunk c (queries 8c..8c+7 of a 64-query half)
    // sits at position c ^ (k % 8) (128-byte swizzle)
    const uint32_t ds_row0 = s_ds + (k >> 3) * 1024 + (k & 7) * 128;
    bool ok = true;
    for (int it = 0; ok && it < nq; ++it) {
      const int st = it % kStages;
      const int qi = i0 + it;
      const bool diag = kCausal && qi == jt;  // keys after a query are masked
      if (!warp_wait(bar_s(qh), it & 1, abort_flag, p.err)) { ok = false; break; }
      // (the stage's LSE / Delta vectors came by TMA: observe their barrier too)
      if (!warp_wait(bar_qfull(st), (it / kStages) & 1, abort_flag, p.err)) { ok = false; break; }
      tc_fence_after();
      const float* lse2 = reinterpret_cast<const float*>(smem + kSmemVec + st * 2 * kBM * 4);
      const uint32_t ds_row = ds_row0 + (it & 1) * (2 * kTile);  // dS buffer of this tile
      const float* dlt = lse2 + kBM;
      const int c = gq;  // this warp's 32-query chunk, in two 16-query parts
#pragma unroll 1
      for (int u = 0; u < 2; ++u) {
        uint32_t sr[16], dpr[16];
        tmem_ld16_nowait(tS + 32 * c + 16 * u, sr);
        tmem_ld16_nowait(tDP + 32 * c + 16 * u, dpr);
        tmem_wait_ld16_dep(sr);
        tmem_wait_ld16_dep(dpr);
        uint32_t pk_p[8], pk_ds[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int q0 = 32 * c + 16 * u + 2 * e;
          const float2 l2 = *reinterpret_cast<const float2*>(lse2 + q0);
          const float2 d2 = *reinterpret_cast<const float2*>(dlt + q0);
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1])),
                                      scl2, make_float2(-l2.x, -l2.y));
          // (all on the MUFU: moving 2/8 or 4/8 of the pairs to the FMA-pipe
          // exp2 measured slower here)
          float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          if (diag) {
            pp.x = (k > q0) ? 0.0f : pp.x;
            pp.y = (k > q0 + 1) ? 0.0f : pp.y;
          }
          const float2 g = __fadd2_rn(make_float2(__uint_as_float(dpr[2 * e]), __uint_as_float(dpr[2 * e + 1])),
                                      make_float2(-d2.x, -d2.y));
          const float2 ds = __fmul2_rn(pp, g);
          pk_p[e] = pack_f16x2(pp.x, pp.y);
          pk_ds[e] = pack_f16x2(ds.x, ds.y);
        }
        // P^T and dS^T into columns this warp has read: queries 32c + 16u..
        // at column 32c + 8u
        tmem_st8(tS + 32 * c + 8 * u, pk_p);
        tmem_st8(tDP + 32 * c + 8 * u, pk_ds);
        // dS^T row k, queries 32c + 16u ..: half c / 2, chunks 4 (c % 2) + 2u, +1
        const uint32_t half = ds_row + (c >> 1) * (kTile);
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          const int ch = 4 * (c & 1) + 2 * u + v;
          st_shared_v4(half + ((ch ^ (k & 7)) << 4), pk_ds[4 * v], pk_ds[4 * v + 1], pk_ds[4 * v + 2],
                       pk_ds[4 * v + 3]);
        }
      }
      tmem_st_wait();
      fence_proxy_async_smem();  // dS in shared memory is read by the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p(qh));
    }
    // ---- dK, dV epilogue (warpgroups 0, 1 write dV, 2, 3 dK; 32 columns each) ----
    if (ok) ok = warp_wait(bar_final, 0, abort_flag, p.err);
    const int key = kv_start + k;
    if (ok && !*abort_flag) {
      tc_fence_after();
      const long long rowoff =
          (p.bnhd ? (static_cast<long long>(b) * p.n + key) * p.nh + h
                  : static_cast<long long>(bh) * p.n + key) * kD;
      {
        const int which = gq >> 1;   // 0: dV, 1: dK
        const int colh = gq & 1;     // columns 32 colh .. 32 colh + 31
        uint32_t r[32];
        const uint32_t col = tmem + lane_base + (which ? kColDK : kColDV) + 32 * colh;
        tmem_ld32_wait(col, r);
        const float f = which ? p.scale : 1.0f;
        if (key < p.n) {
          uint4* dst = reinterpret_cast<uint4*>((which ? p.dk : p.dv) + rowoff + 32 * colh);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            dst[c] = make_uint4(
                pack_f16x2(__uint_as_float(r[8 * c + 0]) * f, __uint_as_float(r[8 * c + 1]) * f),
                pack_f16x2(__uint_as_float(r[8 * c + 2]) * f, __uint_as_float(r[8 * c + 3]) * f),
                pack_f16x2(__uint_as_float(r[8 * c + 4]) * f, __uint_as_float(r[8 * c + 5]) * f),
                pack_f16x2(__uint_as_float(r[8 * c + 6]) * f, __uint_as_float(r[8 * c + 7]) * f));
        }
      }
    }
  } else if (warp >= 20) {
    // ======================= dQ drain (one thread per query row) =======================
    const int t = threadIdx.x - 640;
    const uint32_t tQ = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + kColDQ;
    // staging: two [128 x 32] fp32 halves with the 128-byte swizzle of the
    // dQ tensor map (16-byte chunk c of row t at position c ^ (t % 8))
    uint8_t* srow = smem + kSmemDQ + t * 128;
    bool ok = true;
    for (int it = 0; ok && it < nq; ++it) {
      if (!warp_wait(bar_mm, it & 1, abort_flag, p.err)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // 32 columns at a time
        uint32_t r[32];
        tmem_ld32_wait(tQ + 32 * hh, r);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const int c = 8 * hh + cc;
          const float4 v = make_float4(__uint_as_float(r[4 * cc]) * p.scale, __uint_as_float(r[4 * cc + 1]) * p.scale,
                                       __uint_as_float(r[4 * cc + 2]) * p.scale,
                                       __uint_as_float(r[4 * cc + 3]) * p.scale);
          *reinterpret_cast<float4*>(srow + (c >> 3) * (kBM * 128) + (((c & 7) ^ (t & 7)) << 4)) = v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_dqfree);
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (t == 0) {
        tma_reduce_add_4d(&p.tm_dq, s_dq, 0, (i0 + it) * kBM, h, b);
        tma_reduce_add_4d(&p.tm_dq, s_dq + kBM * 128, 32, (i0 + it) * kBM, h, b);
        tma_store_commit();
        tma_store_wait_read0();  // staging tile reusable
      }
      named_bar_sync(1, 128);
    }
    if (t == 0) tma_store_wait0();  // the adds have landed before the CTA ends
  }
  // warps 2 and 3 have no role

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Delta = rowsum(dO * O) and lse2 = LSE * log2(e) per query row, padded to
// whole 128-row tiles (Delta 0 and lse2 +inf past N: those rows get p = 0).
// Eight threads per row, 16 bytes of O and dO each. LSE is [B, H, N] in
// either layout.
__global__ void flash2_bwd_prep_kernel(const __half* __restrict__ o, const __half* __restrict__ dout,
                                       const float* __restrict__ lse, float* __restrict__ lse2,
                                       float* __restrict__ delta, int n, int npad, long long rows,
                                       int nh, int bnhd) {
  // the main kernel may start its set-up now (it waits for this grid's writes)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = gid >> 3;
  const int sub = threadIdx.x & 7;
  const bool valid_row = row < rows;
  const long long bh = valid_row ? row / npad : 0;
  const int r = valid_row ? static_cast<int>(row - bh * npad) : 0;
  float d = 0.0f;
  if (valid_row && r < n) {
    const long long row_elem = bnhd ? ((bh / nh) * n + r) * nh + bh % nh : bh * n + r;
    const long long off = row_elem * kD + sub * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(o + off);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + off);
    const __half2* ah = reinterpret_cast<const __half2*>(&a);
    const __half2* gh = reinterpret_cast<const __half2*>(&g);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = __half22float2(ah[e]);
      const float2 y = __half22float2(gh[e]);
      d = fmaf(x.x, y.x, d);
      d = fmaf(x.y, y.y, d);
    }
  }
  d += __shfl_xor_sync(0xffffffffu, d, 4);
  d += __shfl_xor_sync(0xffffffffu, d, 2);
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  if (valid_row && sub == 0) {
    delta[row] = d;
    lse2[row] = (r < n) ? lse[bh * n + r] * 1.4426950408889634f : INFINITY;
  }
}

// fp32 map {64, N, H, B} over the dQ accumulator, laid out like dq itself
// ([B,H,N,64] or, with bnhd, [B,N,H,64]) so the final cast is elementwise.
bool encode_dq_map(CUtensorMap* tm, float* base, int64_t n, int64_t H, int64_t B, bool bnhd) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t row_b = kD * 4;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(n),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {bnhd ? H * row_b : row_b,
                           bnhd ? row_b : static_cast<cuuint64_t>(n) * row_b,
                           static_cast<cuuint64_t>(n) * H * row_b};
  cuuint32_t box[4] = {32, static_cast<cuuint32_t>(kBM), 1, 1};  // 128-byte rows
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kCausal>
cudaError_t launch_bwd_variant(const BwdParams& prm, int grid, cudaStream_t stream) {
  auto kern = flash2_bwd_kernel<kCausal>;
  static std::atomic<bool> configured[kMaxFlagDevices];
  const cudaError_t e = ensure_smem_limit(kern, kSmemAlloc, configured);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, prm);
}

}  // namespace

size_t flash2_bwd_workspace_bytes(int64_t BH, int64_t N) {
  const int64_t npad = (N + kBM - 1) / kBM * kBM;
  return static_cast<size_t>(BH * N * kD + 2 * BH * npad) * sizeof(float);
}

cudaError_t launch_flash2_bwd(const void* q, const void* k, const void* v, const void* o,
                              const void* dout, const float* lse, void* dq, void* dk, void* dv,
                              void* workspace, int64_t B, int64_t H, int64_t N, float sm_scale,
                              bool causal, bool bnhd, cudaStream_t stream, const char** where) {
  const int64_t BH = B * H;
  const int64_t npad = (N + kBM - 1) / kBM * kBM;
  float* dq_acc = static_cast<float*>(workspace);
  float* lse2 = dq_acc + BH * N * kD;
  float* delta = lse2 + BH * npad;
  BwdParams prm;
  std::memset(&prm, 0, sizeof(prm));
  if (!encode_rows_map(&prm.tm_q, q, N, H, B, bnhd, kD, kBM) ||
      !encode_rows_map(&prm.tm_k, k, N, H, B, bnhd, kD, kBK) ||
      !encode_rows_map(&prm.tm_v, v, N, H, B, bnhd, kD, kBK) ||
      !encode_rows_map(&prm.tm_do, dout, N, H, B, bnhd, kD, kBM) ||
      !encode_dq_map(&prm.tm_dq, dq_acc, N, H, B, bnhd)) {
    *where = "tensor map encoding";
    return cudaErrorInvalidValue;
  }
  *where = "dq accumulator clear";
  cudaError_t e = cudaMemsetAsync(dq_acc, 0, sizeof(float) * BH * N * kD, stream);
  if (e != cudaSuccess) return e;
  *where = "preprocess launch";
  const long long rows = BH * npad;
  const int threads = 256;
  const long long blocks = (rows * 8 + threads - 1) / threads;
  flash2_bwd_prep_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const __half*>(o), static_cast<const __half*>(dout), lse, lse2, delta,
      static_cast<int>(N), static_cast<int>(npad), rows, static_cast<int>(H), bnhd ? 1 : 0);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  prm.lse2 = lse2;
  prm.delta = delta;
  prm.dk = static_cast<__half*>(dk);
  prm.dv = static_cast<__half*>(dv);
  prm.err = device_error_word();
  prm.n = static_cast<int>(N);
  prm.npad = static_cast<int>(npad);
  prm.bh = static_cast<int>(BH);
  prm.nh = static_cast<int>(H);
  prm.bnhd = bnhd ? 1 : 0;
  prm.n_tiles = static_cast<int>(npad / kBM);
  prm.scale = sm_scale;
  prm.scale_log2 = static_cast<float>(sm_scale * 1.44269504088896340736);
  const int64_t grid = static_cast<int64_t>(prm.n_tiles) * BH;
  *where = "backward kernel launch";
  if (grid <= 0 || grid > 0x7fffffff) return cudaErrorInvalidConfiguration;
  e = causal ? launch_bwd_variant<true>(prm, static_cast<int>(grid), stream)
             : launch_bwd_variant<false>(prm, static_cast<int>(grid), stream);
  if (e != cudaSuccess) return e;
  *where = "dq conversion launch";
  return launch_ring_finalize(dq_acc, dq, BH * N * kD, stream);
}

}  // namespace fl
