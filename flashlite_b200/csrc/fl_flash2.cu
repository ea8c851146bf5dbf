// FlashAttention-2 forward for B200 (sm_100a), head_dim 64, fp16 in/out.
//
// Same mathematics as the reference kernels flash_attn2_wmma_br64/br128
// (thebigblender/FlashLite csrc/kernel_flash2.cu:54-387, :393-727): scores
// prescaled by sm_scale*log2(e) (:772), online softmax with base-2
// exponentials (:232-347), P rounded to fp16 before the PV product while the
// row sum l accumulates fp32 p (:278-294, :339), fully masked rows produce 0
// (:364-365). The implementation is a new design:
//
//  * one CTA owns one or two 128-row query tiles (Q0, Q1) of one (b,h) slice
//    and streams 128-key K and V tiles through two independent TMA rings
//    (kStagesK / kStagesV deep, 128B-swizzled shared memory). K and V have
//    their own producer warps and are released separately (K after the last
//    S = Q K^T that reads it, V after the last P V), so loads run far ahead
//    of use: a TMA tile load takes several microseconds to land here.
//  * warp 1 issues tcgen05.mma from one elected lane with warp-uniform
//    operands; S and O accumulate in Tensor Memory (TMEM), P is written by
//    the softmax warps into its own TMEM columns and fed as operand A.
//  * warpgroups 1 and 2 run the online softmax of Q0 and Q1, one thread per
//    query row. A softmax warp releases its S columns right after loading
//    them (barrier s_free), so S_{j+1} = Q K_{j+1}^T runs on the tensor core
//    while tile j is still being exponentiated; the only wait left on the
//    softmax path is for P V of the previous tile (its P columns are reused).
//    The two warpgroups run part of a KV tile apart: every SM sub-partition
//    holds one warp of each, and while one waits on a barrier or a TMEM round
//    trip (each costs a few hundred cycles while the other warp keeps the
//    MUFU queue full) the other computes.
//  * O is rescaled only when a row maximum grows by more than 2^8 (O and l
//    always share one reference maximum, so the result is unchanged up to
//    rounding), which removes almost every TMEM round trip of O.
//  * the epilogue normalises O, stages it in shared memory (reusing the Q
//    tile) and writes it with one TMA store per tile (coalesced, 16 KB).
//  * every mbarrier wait is bounded; on timeout the CTA records an error,
//    drains its in-flight copies and MMAs, frees TMEM and returns.
//
// A "merge" instantiation serves ring attention: queries and keys carry
// global position offsets for the causal mask, and the epilogue merges the
// block result into a running (fp32 O, log-sum-exp) state in global memory.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "fl_flash2_common.cuh"
#include "fl_internal.h"
#include "fl_ptx.cuh"

namespace fl {
namespace {

// Optional phase trace (build with -DFL_TRACE; compiled out otherwise):
// CTA 0 records clock64() at pipeline events of its first kTraceIters KV
// tiles into fl_trace_buf[event][iteration] for timeline analysis.
#ifdef FL_TRACE
constexpr int kTraceIters = 64;
constexpr int kTraceEvents = 20;
__device__ long long fl_trace_buf[kTraceEvents * kTraceIters];
#define FL_TRACE_EV(ev, it)                                                        \
  do {                                                                             \
    if (blockIdx.x == 0 && (it) < kTraceIters)                                     \
      fl_trace_buf[(ev) * kTraceIters + (it)] = clock64();                         \
  } while (0)
}  // namespace
// Host read-out of the trace (trace builds only).
extern "C" int fl_trace_read(long long* host, int n) {
  const int total = kTraceEvents * kTraceIters;
  return cudaMemcpyFromSymbol(host, fl_trace_buf, sizeof(long long) * (n < total ? n : total)) == cudaSuccess
             ? 0 : -1;
}
namespace {
#else
#define FL_TRACE_EV(ev, it) \
  do {                      \
  } while (0)
#endif

// kSplit (non-merge launches that would leave SMs idle with one query tile
// per CTA): both query-tile slots of a CTA work on the same tile, slot 0 on
// the first half of its KV tiles and slot 1 on the second half; the two
// partial results are merged in the epilogue.
template <int HD, bool kCausal, bool kMerge, bool kSplit = false>
__global__ void __launch_bounds__(kThreads, 1) flash2_fwd_kernel(const __grid_constant__ Flash2Params p) {
  using C = Cfg<HD>;
  constexpr int kD = C::kD;
  constexpr int kBN = C::kBN;
  constexpr int kStagesK = C::kStagesK;
  constexpr int kStagesV = C::kStagesV;
  constexpr int kQTileBytes = C::kQTileBytes;
  constexpr int kSmemQ = C::kSmemQ;
  constexpr int kSmemMisc = C::kSmemMisc;
  constexpr auto col_s = C::col_s;
  constexpr auto col_o = C::col_o;
  constexpr auto col_p = C::col_p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t s_q[2] = {sbase + kSmemQ, sbase + kSmemQ + kQTileBytes};
  const uint32_t s_k0 = sbase + C::kSmemK;
  const uint32_t s_v0 = sbase + C::kSmemV;
  const uint32_t bar_q = sbase + C::kSmemBar;
  const uint32_t bar_kfull0 = bar_q + 8;
  const uint32_t bar_kempty0 = bar_kfull0 + 8 * kStagesK;
  const uint32_t bar_vfull0 = bar_kempty0 + 8 * kStagesK;
  const uint32_t bar_vempty0 = bar_vfull0 + 8 * kStagesV;
  const uint32_t bar_x0 = bar_vempty0 + 8 * kStagesV;
  auto bar_kfull = [&](int st) { return bar_kfull0 + 8u * st; };
  auto bar_kempty = [&](int st) { return bar_kempty0 + 8u * st; };
  auto bar_vfull = [&](int st) { return bar_vfull0 + 8u * st; };
  auto bar_vempty = [&](int st) { return bar_vempty0 + 8u * st; };
  auto bar_s = [&](int i) { return bar_x0 + 8u * (0 + i); };       // S_i ready in TMEM
  auto bar_sfree = [&](int i) { return bar_x0 + 8u * (2 + i); };   // S_i loaded by softmax
  auto bar_p = [&](int i) { return bar_x0 + 8u * (4 + i); };       // P_i written
  auto bar_pv = [&](int i) { return bar_x0 + 8u * (6 + i); };      // P_i V done (O_i updated)
  const uint32_t bar_drain = bar_x0 + 8u * 8;
  const uint32_t bar_stagger = bar_x0 + 8u * 9;  // tile 0 part-way through its first tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work unit: (cta_m, bh); causal launches the longest rows first ----
  const int lin = blockIdx.x;
  int cta_m, bh;
  if (kCausal) {
    cta_m = p.n_cta_m - 1 - lin / p.bh;
    bh = lin % p.bh;
  } else {
    cta_m = lin % p.n_cta_m;
    bh = lin / p.n_cta_m;
  }
  const int qt0 = cta_m * p.tiles_per_cta;
  // split: slot 0 takes the first ceil(n/2) of the tile's n KV tiles, slot 1 the rest
  const int nkv_split = kSplit ? kv_tiles_for<kBN>(p, kCausal, qt0 * kBM) : 0;
  const bool has_q1 = kSplit ? (nkv_split > 1) : ((p.tiles_per_cta == 2) && (qt0 + 1 < p.n_qtiles));
  const int nkv0 = kSplit ? (nkv_split + 1) / 2 : kv_tiles_for<kBN>(p, kCausal, qt0 * kBM);
  const int nkv1 = kSplit ? nkv_split - nkv0
                          : (has_q1 ? kv_tiles_for<kBN>(p, kCausal, (qt0 + 1) * kBM) : 0);
  const int kvb1 = kSplit ? nkv0 : 0;  // first KV tile of slot 1
  const int nkv = nkv0 > nkv1 ? nkv0 : nkv1;

  // ---- setup ----
  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int st = 0; st < kStagesK; ++st) {
      mbar_init(bar_kfull(st), 1);
      mbar_init(bar_kempty(st), 1);
    }
    for (int st = 0; st < kStagesV; ++st) {
      mbar_init(bar_vfull(st), 1);
      mbar_init(bar_vempty(st), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_s(i), 1);
      mbar_init(bar_sfree(i), 4);  // one arrival per softmax warp
      mbar_init(bar_p(i), 4);
      mbar_init(bar_pv(i), 1);
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_stagger, 4);
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
  // Programmatic dependent launch (the launch allows it): the next kernel on
  // this stream may start its own set-up on SMs this grid leaves idle (the
  // last wave's), and this grid touches global memory only after the
  // previous kernel's writes are visible. Every bounded wait starts after it.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Register split: warpgroup 0 (K producer, MMA, V producer, idle) gives
  // registers to the softmax warpgroups. Each role's code sits inside the
  // branch of its own setmaxnreg so the compiler allocates it against that
  // budget (Cfg::kRegsProducer / kRegsSoftmax).
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(C::kRegsProducer));
  if (warp == 0) {
    // ======================= Q + K producer =======================
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_k);
      mbar_arrive_expect_tx(bar_q, ((has_q1 && !kSplit) ? 2 : 1) * kQTileBytes);
#pragma unroll
      for (int hh = 0; hh < C::kHalves; ++hh) {
        tma_load_4d(s_q[0] + hh * (kBM * 128), &p.tm_q, bar_q, 64 * hh, qt0 * kBM, bh % p.nh,
                    bh / p.nh);
        if (has_q1 && !kSplit)
          tma_load_4d(s_q[1] + hh * (kBM * 128), &p.tm_q, bar_q, 64 * hh, (qt0 + 1) * kBM,
                      bh % p.nh, bh / p.nh);
      }
    }
    __syncwarp();
    const int issued =
        kSplit ? produce_ring_split<HD, kStagesK>(&p.tm_k, s_k0, bar_kfull0, bar_kempty0, nkv0, nkv1, kvb1,
                                                  bh % p.nh, bh / p.nh, lane, abort_flag, p.err)
               : produce_ring<HD, kStagesK>(&p.tm_k, s_k0, bar_kfull0, bar_kempty0, nkv, bh % p.nh,
                                            bh / p.nh, lane, abort_flag, p.err);
    if (*abort_flag && lane == 0) {
      // Drain: let every copy this CTA started land before shared memory is released.
      mbar_wait_quiet(bar_q, 0);
      drain_ring<kStagesK>(bar_kfull0, issued);
    }
  } else if (warp == 2) {
    // ======================= V producer =======================
    if (lane == 0) tma_prefetch_desc(&p.tm_v);
    const int issued =
        kSplit ? produce_ring_split<HD, kStagesV>(&p.tm_v, s_v0, bar_vfull0, bar_vempty0, nkv0, nkv1, kvb1,
                                                  bh % p.nh, bh / p.nh, lane, abort_flag, p.err)
               : produce_ring<HD, kStagesV>(&p.tm_v, s_v0, bar_vfull0, bar_vempty0, nkv, bh % p.nh,
                                            bh / p.nh, lane, abort_flag, p.err);
    if (*abort_flag && lane == 0) drain_ring<kStagesV>(bar_vfull0, issued);
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    constexpr uint32_t idesc_s = make_idesc_f16_f32(kBM, kBN, false);  // K-major A and B
    constexpr uint32_t idesc_pv = make_idesc_f16_f32(kBM, kD, true);   // B (= V) MN-major
    // The whole warp runs this code with identical values, so the compiler
    // keeps every MMA operand in uniform registers; one elected lane issues.
    // (Operands built in lane-0-only code cost ~100 cycles per tcgen05.mma.)
    // Descriptors advance by constants: +32 B per K step inside a 128B-swizzled
    // K-major row (encoded +2), to the next 64-column half block after four
    // K steps (D = 128), +2048 B per 16 keys of MN-major V (encoded +128); V's
    // two 64-column halves (D = 128) are one leading-byte-offset apart.
    const uint32_t tm = __shfl_sync(0xffffffffu, tmem, 0);
    const uint64_t dq0 = make_sdesc_sw128(s_q[0], 16, 1024);
    const uint64_t dq1 = make_sdesc_sw128(s_q[1], 16, 1024);
    const uint64_t dk0 = make_sdesc_sw128(s_k0, 16, 1024);
    const uint64_t dv0 = make_sdesc_sw128(s_v0, HD == 64 ? 8192 : kBN * 128, 1024);
    constexpr uint64_t kStageEnc = C::kKVTileBytes >> 4;  // one stage in descriptor units
    constexpr uint64_t kQHalfEnc = (kBM * 128) >> 4;      // Q half block
    constexpr uint64_t kKHalfEnc = (kBN * 128) >> 4;      // K half block
    auto issue_s = [&](int i, int st) {
      const uint64_t a = (i && !kSplit) ? dq1 : dq0;
      const uint64_t b = dk0 + static_cast<uint64_t>(st) * kStageEnc;
      const uint32_t d = tm + col_s(i);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_f16_ss(d, a + 2 * (kk & 3) + (kk >> 2) * kQHalfEnc, b + 2 * (kk & 3) + (kk >> 2) * kKHalfEnc,
                      idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(bar_s(i));
      }
      __syncwarp();
    };
    auto issue_pv = [&](int i, int st, int j) {
      const uint64_t b = dv0 + static_cast<uint64_t>(st) * kStageEnc;
      const uint32_t d = tm + col_o(i);
      const uint32_t a = tm + col_p(i);
      const uint32_t acc0 = j > 0 ? 1u : 0u;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_f16_ts(d, a + kk * 8, b + 128 * kk, idesc_pv, kk > 0 ? 1u : acc0);
        umma_commit(bar_pv(i));
      }
      __syncwarp();
    };
    auto commit_to = [&](uint32_t bar) {
      if (elect_one()) umma_commit(bar);
      __syncwarp();
    };

    // Ring index of slot i's KV step j: j, or 2j + i when the two slots
    // stream different KV tiles through one ring (split).
    auto ring = [&](int i, int j) { return kSplit ? 2 * j + i : j; };
    bool ok = warp_wait_issuer(bar_q, 0, abort_flag, p.err);
    if (ok && nkv > 0) ok = warp_wait_issuer(bar_kfull(0), 0, abort_flag, p.err);
    if (ok && kSplit && nkv1 > 0) ok = warp_wait_issuer(bar_kfull(1), 0, abort_flag, p.err);
    if (ok && nkv > 0) {
      tc_fence_after();
      if (nkv0 > 0) issue_s(0, 0);
      if (kSplit) commit_to(bar_kempty(0));
      if (nkv1 > 0) issue_s(1, ring(1, 0));
      if (!kSplit || nkv1 > 0) commit_to(bar_kempty(ring(1, 0)));
      // Issue order per iteration j, matching the staggered softmax tiles
      // (tile 1 runs part of a KV step behind tile 0): S_0(j+1),
      // P_1(j-1) V, S_1(j+1), P_0(j) V. Each MMA waits only for its own
      // inputs, so neither tile's softmax waits behind the other's.
      for (int j = 0; j <= nkv; ++j) {
        if (lane == 0) FL_TRACE_EV(19, j);
        const bool s_next = j + 1 < nkv;
        const int rk0 = ring(0, j + 1);
        const int sk = rk0 % kStagesK;
        if (s_next) {
          if (!warp_wait_issuer(bar_kfull(sk), (rk0 / kStagesK) & 1, abort_flag, p.err)) break;
          if (lane == 0) FL_TRACE_EV(10, j);
        }
        if (j + 1 < nkv0) {
          if (!warp_wait_issuer(bar_sfree(0), j & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_s(0, sk);
          if (kSplit) commit_to(bar_kempty(sk));  // that K tile is read by S_0 only
          if (lane == 0) FL_TRACE_EV(12, j);
        }
        if (j >= 1) {
          // P_1 V of the previous KV tile, then that V stage is free.
          const int rv1 = ring(1, j - 1);
          const int sv = rv1 % kStagesV;
          if (j - 1 < nkv1) {
            // (split: slot 1's V tile is its own ring entry, not yet waited for)
            if (kSplit && !warp_wait_issuer(bar_vfull(sv), (rv1 / kStagesV) & 1, abort_flag, p.err)) break;
            if (!warp_wait_issuer(bar_p(1), (j - 1) & 1, abort_flag, p.err)) break;
            tc_fence_after();
            if (lane == 0) FL_TRACE_EV(9, j - 1);
            issue_pv(1, sv, j - 1);
            if (lane == 0) FL_TRACE_EV(13, j - 1);
          }
          if (!kSplit || j - 1 < nkv1) commit_to(bar_vempty(sv));
        }
        const int rk1 = ring(1, j + 1);
        const int sk1 = rk1 % kStagesK;
        if (j + 1 < nkv1) {
          if (kSplit && !warp_wait_issuer(bar_kfull(sk1), (rk1 / kStagesK) & 1, abort_flag, p.err)) break;
          if (!warp_wait_issuer(bar_sfree(1), j & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_s(1, sk1);
          if (lane == 0) FL_TRACE_EV(18, j);
        }
        if (kSplit ? (j + 1 < nkv1) : s_next) commit_to(bar_kempty(sk1));
        if (j < nkv) {
          // V_j must be resident for P_0 V (and later P_1 V).
          const int rv0 = ring(0, j);
          const int sv = rv0 % kStagesV;
          if (!warp_wait_issuer(bar_vfull(sv), (rv0 / kStagesV) & 1, abort_flag, p.err)) break;
          if (j < nkv0) {
            if (!warp_wait_issuer(bar_p(0), j & 1, abort_flag, p.err)) break;
            tc_fence_after();
            if (lane == 0) FL_TRACE_EV(8, j);
            issue_pv(0, sv, j);
            if (lane == 0) FL_TRACE_EV(11, j);
          }
          if (kSplit) commit_to(bar_vempty(sv));  // that V tile is read by P_0 V only
        }
      }
    }
    // Drain: wait until every MMA this thread issued has completed.
    if (elect_one()) {
      umma_commit(bar_drain);
      mbar_wait_quiet(bar_drain, 0);
    }
    __syncwarp();
  }
  // warp 3 has no role in this design.
  } else {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(C::kRegsSoftmax));
  {
    // ======================= softmax warpgroups =======================
    const int i = (warp - 4) >> 2;               // query tile handled: 0 or 1
    const int t = threadIdx.x - 128 * (1 + i);   // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t tS = tmem + lane_base + col_s(i);
    const uint32_t tP = tmem + lane_base + col_p(i);
    const uint32_t tO = tmem + lane_base + col_o(i);
    const int q_start = (qt0 + (kSplit ? 0 : i)) * kBM;
    const int my_nkv = (i == 0) ? nkv0 : nkv1;
    const int kv_base = (i == 0) ? 0 : kvb1;  // first KV tile of this slot
    const bool active = (i == 0) || has_q1;

    float sc = p.scale_log2;
    const bool prescale = !(sc > 0.0f);  // negative scales: scale before max/mask
    float m_ref = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    // The two tiles run part of a KV step apart, so that one warp of each SM
    // sub-partition computes while the other waits on a barrier or a TMEM
    // round trip: tile 0 signals part-way through its first tile and tile 1
    // starts then.
    bool stagger_sent = (i != 0);
    if (i == 1 && my_nkv > 0) ok = warp_wait(bar_stagger, 0, abort_flag, p.err);

    for (int j = 0; ok && j < my_nkv; ++j) {
      if (t == 0 && i == 0) FL_TRACE_EV(19, j);
      if (!warp_wait(bar_s(i), j & 1, abort_flag, p.err)) { ok = false; break; }
      if (t == 0) FL_TRACE_EV(0 + 4 * i, j);
      tc_fence_after();
      uint32_t sr[kBN];
      if constexpr (kBN == 128) {
        tmem_ld128_wait(tS, sr);
      } else {
        tmem_ld64_wait(tS, sr);
      }
      // S_i is in registers: let the tensor core overwrite it with S_{i,j+1}.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree(i));
      if (t == 0) FL_TRACE_EV(1 + 4 * i, j);
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN; ++c) s[c] = __uint_as_float(sr[c]);
      float scl = sc;
      if (prescale) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) s[c] *= sc;
        scl = 1.0f;
      }
      const int k_start = (j + kv_base) * kBN;
      // keys visible to this row: c < limit
      long long lim = p.nk - k_start;
      if (kCausal) {
        const long long d = p.q_offset + q_start + t - (p.kv_offset + k_start) + 1;
        lim = d < lim ? d : lim;
      }
      if (lim < kBN) {
        const int limit = lim < 0 ? 0 : static_cast<int>(lim);
#pragma unroll
        for (int c = 0; c < kBN; ++c) s[c] = (c < limit) ? s[c] : -INFINITY;
      }
      // Row maximum, kept separately over the columns exponentiated on the
      // FMA pipe (mxp) and on the MUFU (mxm): 3-input max chains, several
      // independent per class (no 127-long dependency chain).
      float mxp, mxm;
      {
        constexpr int kNP = poly_cols(kBN), kNM = kBN - kNP;  // per row
        float vp[kNP], vm[kNM];
        int np = 0, nm = 0;
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          const int e = (c >> 1) & 15;
          if ((kPolyPairs >> (e & 7)) & 1) {
            vp[np++] = s[c];
            vp[np++] = s[c + 1];
          } else {
            vm[nm++] = s[c];
            vm[nm++] = s[c + 1];
          }
        }
        mxp = max_chains4<kNP>(vp);
        mxm = max_chains4<kNM>(vm);
      }
      const float mx = fmaxf(mxp, mxm);
      if (t == 0) FL_TRACE_EV(2 + 4 * i, j);
      const float m_tile = mx * scl;
      const float m_new = fmaxf(m_ref, m_tile);
      const bool need = m_new > m_ref + kRescaleThreshold;
      float alpha = 1.0f;
      if (need) {
        alpha = ex2_approx(m_ref - m_new);
        m_ref = m_new;
      }
      l *= alpha;
      // P V of the previous tile must be done before its P columns are
      // rewritten and before O is rescaled.
      auto wait_pv_rescale = [&]() -> bool {
        if (j == 0) return true;
        if (!warp_wait(bar_pv(i), (j - 1) & 1, abort_flag, p.err)) return false;
        tc_fence_after();
        if (t == 0) FL_TRACE_EV(16 + i, j);
        if (__any_sync(0xffffffffu, need)) {
          uint32_t o[32];
#pragma unroll
          for (int h = 0; h < kD / 32; ++h) {
            tmem_ld32_wait(tO + h * 32, o);
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(tO + h * 32, o);
          }
        }
        return true;
      };
      // Split-KV CTAs (head_dim 64) compute the step's exponentials before
      // this wait and store P after it, so the wait overlaps them: config 2
      // 322 -> 340 TF/s, config 2 causal 154 -> 164. In the two-tile
      // instantiations the same order makes ptxas spill (216 bytes reloaded
      // per step) and costs 3-9 %, so they wait first.
      constexpr bool kExpFirst = kSplit && HD == 64;
      if (!kExpFirst && !wait_pv_rescale()) { ok = false; break; }
      const float m_use = (m_ref == -INFINITY) ? 0.0f : m_ref;
      // p = 2^(s*scale - m_use): packed fp32x2 FMA for the argument, MUFU ex2,
      // fp16x2 pack for the PV operand; l sums the unrounded p in four
      // independent packed partial sums.
      const float2 scl2 = make_float2(scl, scl);
      const float2 nm2 = make_float2(-m_use, -m_use);
      float2 lsum[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int q = 0; q < kBN / 32; ++q) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int c = q * 32 + 2 * e;
          const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), scl2, nm2);
          // Column pairs in kPolyPairs take the FMA-pipe exp2; the rest the
          // MUFU. Splitting the work keeps both pipes busy.
          const float2 pp = ((kPolyPairs >> (e & 7)) & 1)
                                ? exp2_poly2(x)
                                : make_float2(ex2_approx(x.x), ex2_approx(x.y));
          lsum[e & 3] = __fadd2_rn(lsum[e & 3], pp);
          pk[q * 16 + e] = pack_f16x2(pp.x, pp.y);
        }
        if (!kExpFirst) tmem_st16(tP + q * 16, *reinterpret_cast<const uint32_t(*)[16]>(&pk[q * 16]));
        // Tile 1 starts when tile 0 is three quarters through its first KV
        // tile (128-key tiles; half-way with 64-key tiles): measured ~1 %
        // faster than half-way on the config-3 shapes, same output bits.
        if (q == (kBN == 128 ? 2 : 0) && !stagger_sent) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_stagger);
          stagger_sent = true;
        }
      }
      {
        const float2 a = __fadd2_rn(lsum[0], lsum[1]);
        const float2 b = __fadd2_rn(lsum[2], lsum[3]);
        l += (a.x + a.y) + (b.x + b.y);
        // The tile's largest p enters O through its fp16 rounding; let l see
        // the same value so a row dominated by one key reproduces that key's
        // V row exactly (the reference gets this for free since its running
        // maximum is always exact, csrc/kernel_flash2.cu:250-264).
        // Recompute that p with the method its column used.
        const float xm = fmaf(mx, scl, -m_use);
        const float pm = (mxp >= mxm) ? exp2_poly2(make_float2(xm, xm)).x : ex2_approx(xm);
        l += __half2float(__float2half_rn(pm)) - pm;
      }
      if (kExpFirst) {
        if (!wait_pv_rescale()) { ok = false; break; }
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q)
          tmem_st16(tP + q * 16, *reinterpret_cast<const uint32_t(*)[16]>(&pk[q * 16]));
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p(i));
      if (t == 0) FL_TRACE_EV(3 + 4 * i, j);
      if (t == 96) FL_TRACE_EV(14 + i, j);
    }

    if (!stagger_sent) {  // tile 0 without KV tiles, or stopped early
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_stagger);
    }

    // ---- epilogue ----
    if (active && my_nkv > 0 && ok) ok = warp_wait(bar_pv(i), (my_nkv - 1) & 1, abort_flag, p.err);
    const bool do_out = active && my_nkv > 0 && ok;
    uint32_t o[kD];
    if (do_out) {
      tc_fence_after();
      uint32_t tmp[32];
#pragma unroll
      for (int h = 0; h < kD / 32; ++h) {
        tmem_ld32_wait(tO + h * 32, tmp);
#pragma unroll
        for (int c = 0; c < 32; ++c) o[32 * h + c] = tmp[c];
      }
    }
    if constexpr (kSplit) {
      // Slot 1 hands its row (max, sum) to slot 0 through its unused Q
      // buffer; slot 0 reads slot 1's O from TMEM (same lanes) and merges:
      // O = (O0 2^(m0-m) + O1 2^(m1-m)) / (l0 2^(m0-m) + l1 2^(m1-m)).
      float2* xch = reinterpret_cast<float2*>(smem + kSmemQ + kQTileBytes);
      if (i == 1) xch[t] = make_float2(do_out ? m_ref : -INFINITY, do_out ? l : 0.0f);
      named_bar_sync(3, 256);
      if (i == 0 && do_out) {
        const float2 ml1 = xch[t];
        const float m = fmaxf(m_ref, ml1.x);
        const float w0 = (m_ref == -INFINITY) ? 0.0f : ex2_approx(m_ref - m);
        const float w1 = (ml1.x == -INFINITY) ? 0.0f : ex2_approx(ml1.x - m);
        l = l * w0 + ml1.y * w1;
        m_ref = m;
        if (__any_sync(0xffffffffu, ml1.x != -INFINITY)) {
          uint32_t tmp[32];
#pragma unroll
          for (int h = 0; h < kD / 32; ++h) {
            tmem_ld32_wait(tmem + lane_base + col_o(1) + h * 32, tmp);
#pragma unroll
            for (int c = 0; c < 32; ++c)
              o[32 * h + c] = __float_as_uint(fmaf(__uint_as_float(o[32 * h + c]), w0,
                                                   __uint_as_float(tmp[c]) * w1));
          }
        } else {
#pragma unroll
          for (int c = 0; c < kD; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * w0);
        }
      }
    }
    const float inv_l = (l > 0.0f) ? 1.0f / l : 0.0f;
    if (!kMerge) {
      // A tile whose rows see no key at all (key positions offset past the
      // queries) is written as zeros, as fully masked rows are. (Split:
      // slot 0 writes the merged tile.)
      const bool write = active && ok && !(kSplit && i == 1);
      if (write && !do_out) {
        // The staging buffer is this tile's Q buffer: let its load land first
        // (with no KV step nothing else waited for it).
        warp_wait(bar_q, 0, abort_flag, p.err);
#pragma unroll
        for (int c = 0; c < kD; ++c) o[c] = 0u;
      }
      if (p.lse != nullptr && write && q_start + t < p.nq)
        p.lse[static_cast<long long>(bh) * p.nq + q_start + t] =
            (l > 0.0f) ? (m_ref + log2f(l)) * 0.69314718055994531f : -INFINITY;
      if (write) {
        // Stage the fp16 tile in the (now unused) Q buffer with the 128B
        // swizzle the TMA store expects: 16-byte chunk c of row t goes to
        // chunk position c % 8 ^ (t % 8) of half block c / 8.
        uint8_t* row = smem + kSmemQ + i * kQTileBytes + t * 128;
#pragma unroll
        for (int c = 0; c < kD / 8; ++c) {
          uint4 v;
          v.x = pack_f16x2(__uint_as_float(o[8 * c + 0]) * inv_l, __uint_as_float(o[8 * c + 1]) * inv_l);
          v.y = pack_f16x2(__uint_as_float(o[8 * c + 2]) * inv_l, __uint_as_float(o[8 * c + 3]) * inv_l);
          v.z = pack_f16x2(__uint_as_float(o[8 * c + 4]) * inv_l, __uint_as_float(o[8 * c + 5]) * inv_l);
          v.w = pack_f16x2(__uint_as_float(o[8 * c + 6]) * inv_l, __uint_as_float(o[8 * c + 7]) * inv_l);
          *reinterpret_cast<uint4*>(row + (c >> 3) * (kBM * 128) + (((c & 7) ^ (t & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
      }
      named_bar_sync(1 + i, 128);
      if (write && t == 0 && !*abort_flag) {
#pragma unroll
        for (int hh = 0; hh < C::kHalves; ++hh)
          tma_store_4d(&p.tm_o, s_q[i] + hh * (kBM * 128), 64 * hh, q_start, bh % p.nh, bh / p.nh);
        tma_store_commit();
        tma_store_wait_read0();
      }
    } else {
      const int row = q_start + t;
      if (active && (do_out || (p.first && my_nkv == 0 && ok))) {  // warp-uniform
        const bool valid = row < p.nq;
        // ln(sum_j exp(s_j*scale)) = (m_ref + log2(l)) * ln(2)
        const float lse_blk = (l > 0.0f) ? (m_ref + log2f(l)) * 0.69314718055994531f : -INFINITY;
        float* lrow = p.lse + static_cast<long long>(bh) * p.nq + row;
        float w_old = 0.0f, w_new = 1.0f, lse_out = lse_blk;
        if (!p.first) {
          const float lse_old = valid ? *lrow : -INFINITY;
          const float mx = fmaxf(lse_old, lse_blk);
          if (mx == -INFINITY) {
            w_old = 0.0f; w_new = 0.0f; lse_out = -INFINITY;
          } else {
            const float a = __expf(lse_old - mx), b = __expf(lse_blk - mx);
            const float sum = a + b;
            w_old = a / sum; w_new = b / sum;
            lse_out = mx + __logf(sum);
          }
        } else if (lse_blk == -INFINITY) {
          w_new = 0.0f;
        }
        const float wn = w_new * inv_l;
        if (do_out) {
          // Coalesced read-modify-write of the fp32 state. Each warp stages its
          // 32 rows in its quarter of this tile's Q buffer (free: every S MMA
          // of the tile completed before its last P V), kCols columns per
          // pass, 16-byte chunk c of row r at chunk c ^ (r % kCh) so that
          // neither the row-wise writes nor the column-wise reads conflict,
          // then reads and writes 32 / kCh whole rows per instruction.
          constexpr int kCols = kQTileBytes / 4 / (32 * 4);  // 32 (D = 64) or 64 (D = 128)
          constexpr int kCh = kCols / 4;                     // 16-byte chunks per staged row
          constexpr int kRowsPer = 32 / kCh;                 // rows per warp instruction
          float4* stg = reinterpret_cast<float4*>(smem + kSmemQ + i * kQTileBytes + (warp & 3) * (kQTileBytes / 4));
          const int row0 = q_start + (warp & 3) * 32;  // the warp's first row
          constexpr int kIt = 32 / kRowsPer;       // row groups per pass
          constexpr int kPre = kD == 64 ? 2 : 1;   // passes whose old state is loaded at once
          const int c = lane & (kCh - 1);
#pragma unroll
          for (int hb = 0; hb < kD / kCols; hb += kPre) {
            // All loads of the old state first, so they are in flight together
            // (and overlap the staging below) instead of one per row group.
            float4 prev[kPre][kIt];
#pragma unroll
            for (int h2 = 0; h2 < kPre; ++h2)
#pragma unroll
              for (int k = 0; k < kIt; ++k) {
                const int r = k * kRowsPer + lane / kCh;
                prev[h2][k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (!p.first && row0 + r < p.nq)
                  prev[h2][k] = reinterpret_cast<const float4*>(
                      p.o_acc + (static_cast<long long>(bh) * p.nq + row0 + r) * kD + (hb + h2) * kCols)[c];
              }
#pragma unroll
            for (int h2 = 0; h2 < kPre; ++h2) {
              const int hf = hb + h2;
#pragma unroll
              for (int cc = 0; cc < kCh; ++cc) {
                const int e = hf * kCols + 4 * cc;
                stg[lane * kCh + (cc ^ (lane & (kCh - 1)))] =
                    make_float4(__uint_as_float(o[e]) * wn, __uint_as_float(o[e + 1]) * wn,
                                __uint_as_float(o[e + 2]) * wn, __uint_as_float(o[e + 3]) * wn);
              }
              __syncwarp();
#pragma unroll
              for (int k = 0; k < kIt; ++k) {
                const int r = k * kRowsPer + lane / kCh;
                const float wo = __shfl_sync(0xffffffffu, w_old, r);
                const float4 v = stg[r * kCh + (c ^ (r & (kCh - 1)))];
                if (row0 + r < p.nq) {
                  const float4 pv = prev[h2][k];
                  float4 out = v;
                  if (!p.first) out = make_float4(pv.x * wo + v.x, pv.y * wo + v.y, pv.z * wo + v.z, pv.w * wo + v.w);
                  reinterpret_cast<float4*>(p.o_acc + (static_cast<long long>(bh) * p.nq + row0 + r) * kD +
                                            hf * kCols)[c] = out;
                }
              }
              __syncwarp();
            }
          }
        } else if (valid) {
          // no key visible to this tile (first block only): the state starts at zero
          float4* orow = reinterpret_cast<float4*>(p.o_acc + (static_cast<long long>(bh) * p.nq + row) * kD);
#pragma unroll
          for (int c = 0; c < kD / 4; ++c) orow[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (valid) *lrow = lse_out;
      }
    }
  }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  });
  return fn;
}

// Tensor map {D, rows, H, B} over a [B,H,rows,D] (bnhd = false) or
// [B,rows,H,D] (bnhd = true) fp16 array, box {64, box_rows, 1, 1} (one
// 128-byte swizzle atom wide: a D = 128 tile is copied as two halves).
bool encode_rows_map(CUtensorMap* tm, const void* base, int64_t rows, int64_t H, int64_t B,
                     bool bnhd, int D, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t row_b = static_cast<cuuint64_t>(D) * 2;  // bytes of one fp16 row
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3];
  if (!bnhd) {
    strides[0] = row_b;                                       // next row
    strides[1] = static_cast<cuuint64_t>(rows) * row_b;       // next head
  } else {
    strides[0] = static_cast<cuuint64_t>(H) * row_b;          // next row
    strides[1] = row_b;                                       // next head
  }
  strides[2] = static_cast<cuuint64_t>(rows) * H * row_b;     // next batch entry
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

#ifndef FL_SPLIT_KV
#define FL_SPLIT_KV 1
#endif

template <int HD, bool kCausal, bool kMerge, bool kSplit = false>
cudaError_t launch_variant(const Flash2Params& prm, int grid, cudaStream_t stream) {
  constexpr int kSmemAlloc = Cfg<HD>::kSmemAlloc;
  auto kern = flash2_fwd_kernel<HD, kCausal, kMerge, kSplit>;
  static std::atomic<bool> configured[kMaxFlagDevices];
  const cudaError_t e = ensure_smem_limit(kern, kSmemAlloc, configured);
  if (e != cudaSuccess) return e;
  // Launched with programmatic stream serialization (see griddepcontrol in
  // the kernel): back-to-back calls overlap one's set-up with the previous
  // one's last wave (config 2 262 -> 312 TF/s, config 3 643 -> 658).
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

cudaError_t launch_flash2(const void* q, const void* k, const void* v, void* o_f16, float* o_acc,
                          float* lse, int64_t B, int64_t H, int64_t Nq, int64_t Nk,
                          int64_t q_offset, int64_t kv_offset, float scale_log2, bool causal,
                          bool merge, bool first, bool bnhd, cudaStream_t stream, int head_dim) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorInvalidValue;
  Flash2Params prm;
  const int64_t BH = B * H;
  const int kv_rows = head_dim == 64 ? Cfg<64>::kBN : Cfg<128>::kBN;  // keys per KV tile
  if (!encode_rows_map(&prm.tm_q, q, Nq, H, B, bnhd, head_dim, kBM) ||
      !encode_rows_map(&prm.tm_k, k, Nk, H, B, bnhd, head_dim, kv_rows) ||
      !encode_rows_map(&prm.tm_v, v, Nk, H, B, bnhd, head_dim, kv_rows)) {
    return cudaErrorInvalidValue;
  }
  if (!merge) {
    if (!encode_rows_map(&prm.tm_o, o_f16, Nq, H, B, bnhd, head_dim, kBM)) return cudaErrorInvalidValue;
  } else {
    prm.tm_o = prm.tm_q;
  }
  prm.nh = static_cast<int>(H);
  prm.o_acc = o_acc;
  prm.lse = lse;
  prm.err = device_error_word();
  prm.nq = static_cast<int>(Nq);
  prm.nk = static_cast<int>(Nk);
  prm.bh = static_cast<int>(BH);
  prm.n_qtiles = static_cast<int>((Nq + kBM - 1) / kBM);
  prm.n_ktiles = static_cast<int>((Nk + kv_rows - 1) / kv_rows);
  const int64_t pairs = (prm.n_qtiles + 1) / 2;
  // Two query tiles per CTA keep the tensor core busy while one tile is in
  // softmax; fall back to one tile per CTA when that would leave SMs idle.
  prm.tiles_per_cta = (pairs * BH >= sm_count()) ? 2 : 1;
  prm.n_cta_m = (prm.n_qtiles + prm.tiles_per_cta - 1) / prm.tiles_per_cta;
  prm.q_offset = q_offset;
  prm.kv_offset = kv_offset;
  prm.scale_log2 = scale_log2;
  prm.first = first ? 1 : 0;
  prm.sk_total = 0;
  prm.sk_grid = 0;
  prm.sk_ws = nullptr;
  prm.sk_cnt = nullptr;
  prm.sk_epoch = 0;
  const int64_t grid = static_cast<int64_t>(prm.n_cta_m) * BH;
  if (grid <= 0 || grid > 0x7fffffff) return cudaErrorInvalidConfiguration;
  const int g = static_cast<int>(grid);
  // Non-causal head_dim-64 grids whose last wave would leave SMs idle take
  // the stream-K schedule (fl_flash2_sk.cu) where its cost model says so.
  if (!merge && !causal && head_dim == 64 && prm.tiles_per_cta == 2) {
    bool launched = false;
    const cudaError_t e = launch_flash2_sk(prm, grid, stream, &launched);
    if (launched || e != cudaSuccess) return e;
  }
  // One query tile per CTA leaves the second softmax warpgroup idle: give it
  // the second half of the tile's KV tiles instead (split), when there are
  // at least two.
  if (FL_SPLIT_KV && !merge && prm.tiles_per_cta == 1 && prm.n_ktiles >= 2) {
    if (head_dim == 128)
      return causal ? launch_variant<128, true, false, true>(prm, g, stream)
                    : launch_variant<128, false, false, true>(prm, g, stream);
    return causal ? launch_variant<64, true, false, true>(prm, g, stream)
                  : launch_variant<64, false, false, true>(prm, g, stream);
  }
  if (head_dim == 128) {
    if (merge) {
      return causal ? launch_variant<128, true, true>(prm, g, stream)
                    : launch_variant<128, false, true>(prm, g, stream);
    }
    return causal ? launch_variant<128, true, false>(prm, g, stream)
                  : launch_variant<128, false, false>(prm, g, stream);
  }
  if (merge) {
    return causal ? launch_variant<64, true, true>(prm, g, stream)
                  : launch_variant<64, false, true>(prm, g, stream);
  }
  return causal ? launch_variant<64, true, false>(prm, g, stream)
                : launch_variant<64, false, false>(prm, g, stream);
}

}  // namespace fl
