// FlashAttention-2 forward, stream-K schedule (head_dim 64, non-causal).
//
// The same per-step mathematics as flash2_fwd_kernel (fl_flash2.cu), which
// follows the reference kernels (thebigblender/FlashLite
// csrc/kernel_flash2.cu:54-387, :393-727); only the division of work over
// the SMs differs. A launch of U units (a unit is two 128-row query tiles of
// one (b,h) slice and its n_ktiles KV steps) on G SMs runs in ceil(U / G)
// waves when each CTA owns one unit, so a grid of 1.73 waves leaves 27 % of
// the SMs idle in its second wave. Here the units are laid end to end, U *
// n_ktiles KV steps in all, and CTA c of G runs steps [c S / G, (c+1) S / G):
// up to three segments (the end of a unit the previous CTA started, whole
// units, the start of a unit the next CTA finishes), every SM busy to the end.
//
//  * roles as in flash2_fwd_kernel (warp 0 Q and K loads, warp 1 MMA, warp 2
//    V loads, warpgroups 1 and 2 the softmax of the two tiles). Ring
//    positions and barrier phases run on across segments.
//  * two 32 KB buffers alternate between segments: segment s reads its Q
//    tiles from buffer s % 2 and, after its last S MMA, stages its output
//    there for the TMA store, while the next segment's Q is already loaded
//    into the other buffer. The MMA warp issues the next segment's first S
//    right after the last P_0 V, so tile 0 finds it ready after its epilogue.
//  * a unit cut between CTAs: every piece stores its rows normalised (fp32,
//    column-major: coalesced) with their log2-sum-exp in a workspace; the
//    piece that arrives last (an atomic count per unit and tile, tagged with
//    a launch epoch) merges all pieces in piece order and stores the tile,
//    so the output does not depend on which piece finished last. No CTA ever
//    waits for another.
//  * every mbarrier wait is bounded, as in flash2_fwd_kernel.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "fl_flash2_common.cuh"
#include "fl_internal.h"
#include "fl_ptx.cuh"

#ifndef SK_LOOKAHEAD
#define SK_LOOKAHEAD 0
#endif
#ifndef SK_DEFER_READ
#define SK_DEFER_READ 0
#endif

namespace fl {
namespace {

// Shared-memory map: Cfg<64>'s map (buffer A = its Q tiles, the K and V
// rings, its barriers), then buffer B and the stream-K barriers.
template <int HD>
struct SkCfg {
  using C = Cfg<HD>;
  static constexpr int kSmemBufB = (C::kSmemBytes + 1023) & ~1023;  // 2 tiles
  static constexpr int kSmemBar = kSmemBufB + 2 * C::kQTileBytes;    // q_full[2], x_free[2]
  static constexpr int kSmemFlag = kSmemBar + 4 * 8;                 // merge decision per tile
  static constexpr int kSmemBytes = kSmemFlag + 8;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;
};
static_assert(SkCfg<64>::kSmemAlloc <= 227 * 1024, "stream-K shared memory");

// A CTA's part of one unit: KV steps [k0, k1) of unit u.
struct SkSeg {
  int u, k0, k1;
};

__device__ __forceinline__ SkSeg sk_seg(long long w, long long w_end, int nkv) {
  SkSeg s;
  s.u = static_cast<int>(w / nkv);
  s.k0 = static_cast<int>(w - static_cast<long long>(s.u) * nkv);
  const long long left = w_end - w;
  s.k1 = (left < nkv - s.k0) ? s.k0 + static_cast<int>(left) : nkv;
  return s;
}

// Steps [w_begin, w_end) of this CTA: an even share of the total.
__device__ __forceinline__ void sk_range(const Flash2Params& p, long long* w_begin, long long* w_end) {
  const long long c = blockIdx.x;
  *w_begin = p.sk_total * c / p.sk_grid;
  *w_end = p.sk_total * (c + 1) / p.sk_grid;
}

// CTA whose range holds step x (the inverse of sk_range).
__device__ __forceinline__ int sk_cta_of(const Flash2Params& p, long long x) {
  return static_cast<int>(((x + 1) * p.sk_grid - 1) / p.sk_total);
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) flash2_fwd_sk_kernel(const __grid_constant__ Flash2Params p) {
  using C = Cfg<HD>;
  using SC = SkCfg<HD>;
  constexpr int kD = C::kD;
  constexpr int kBN = C::kBN;
  constexpr int kStagesK = C::kStagesK;
  constexpr int kStagesV = C::kStagesV;
  constexpr int kQTileBytes = C::kQTileBytes;
  constexpr int kSmemMisc = C::kSmemMisc;
  constexpr auto col_s = C::col_s;
  constexpr auto col_o = C::col_o;
  constexpr auto col_p = C::col_p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  // buffer b (0: A, 1: B): Q tiles of the segments s with s % 2 == b, then their output
  auto buf = [&](int b) { return sbase + (b ? SC::kSmemBufB : C::kSmemQ); };
  const uint32_t s_k0 = sbase + C::kSmemK;
  const uint32_t s_v0 = sbase + C::kSmemV;
  const uint32_t bar_kfull0 = sbase + C::kSmemBar + 8;  // Cfg's map: q (unused here) first
  const uint32_t bar_kempty0 = bar_kfull0 + 8 * kStagesK;
  const uint32_t bar_vfull0 = bar_kempty0 + 8 * kStagesK;
  const uint32_t bar_vempty0 = bar_vfull0 + 8 * kStagesV;
  const uint32_t bar_x0 = bar_vempty0 + 8 * kStagesV;
  auto bar_kfull = [&](int st) { return bar_kfull0 + 8u * st; };
  auto bar_kempty = [&](int st) { return bar_kempty0 + 8u * st; };
  auto bar_vfull = [&](int st) { return bar_vfull0 + 8u * st; };
  auto bar_vempty = [&](int st) { return bar_vempty0 + 8u * st; };
  auto bar_s = [&](int i) { return bar_x0 + 8u * (0 + i); };      // S_i ready in TMEM
  auto bar_sfree = [&](int i) { return bar_x0 + 8u * (2 + i); };  // S_i loaded by softmax
  auto bar_p = [&](int i) { return bar_x0 + 8u * (4 + i); };      // P_i written
  auto bar_pv = [&](int i) { return bar_x0 + 8u * (6 + i); };     // P_i V done
  const uint32_t bar_drain = bar_x0 + 8u * 8;
  const uint32_t bar_stagger = bar_x0 + 8u * 9;
  auto bar_qfull = [&](int b) { return sbase + SC::kSmemBar + 8u * b; };        // Q landed in buffer b
  auto bar_xfree = [&](int b) { return sbase + SC::kSmemBar + 8u * (2 + b); };  // buffer b reusable
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
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
      mbar_init(bar_qfull(i), 1);
      mbar_init(bar_xfree(i), 2);  // one arrival per tile per segment
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
  // Programmatic dependent launch, as in flash2_fwd_kernel.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(C::kRegsProducer));
  if (warp == 0) {
    // ======================= Q + K producer =======================
    // Segment s's Q goes to buffer s % 2 once segment s - 2 has released it;
    // K tiles stream on across segments.
    const int nkv = p.n_ktiles;
    long long w, w_end;
    sk_range(p, &w, &w_end);
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_k);
    }
    int kr = 0, seg = 0, q_issued = 0;
    bool ok = true;
    for (; ok && w < w_end; ++seg) {
      const SkSeg sg = sk_seg(w, w_end, nkv);
      w += sg.k1 - sg.k0;
      const int cta_m = sg.u % p.n_cta_m, bh = sg.u / p.n_cta_m;
      const int qt0 = 2 * cta_m;
      const bool q1 = qt0 + 1 < p.n_qtiles;
      const int h = bh % p.nh, b = bh / p.nh;
      const int qb = seg & 1;
      if (seg >= 2 && !warp_wait(bar_xfree(qb), ((seg >> 1) - 1) & 1, abort_flag, p.err)) { ok = false; break; }
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_qfull(qb), (q1 ? 2 : 1) * kQTileBytes);
#pragma unroll
        for (int hh = 0; hh < C::kHalves; ++hh) {
          tma_load_4d(buf(qb) + hh * (kBM * 128), &p.tm_q, bar_qfull(qb), 64 * hh, qt0 * kBM, h, b);
          if (q1)
            tma_load_4d(buf(qb) + kQTileBytes + hh * (kBM * 128), &p.tm_q, bar_qfull(qb), 64 * hh,
                        (qt0 + 1) * kBM, h, b);
        }
      }
      __syncwarp();
      q_issued = seg + 1;
      for (int t = sg.k0; t < sg.k1; ++t, ++kr) {
        const int st = kr % kStagesK;
        const uint32_t ph = (kr / kStagesK) & 1;
        if (!warp_wait(bar_kempty(st), ph ^ 1, abort_flag, p.err)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(bar_kfull(st), C::kKVTileBytes);
#pragma unroll
          for (int hh = 0; hh < C::kHalves; ++hh)
            tma_load_4d(s_k0 + st * C::kKVTileBytes + hh * (kBN * 128), &p.tm_k, bar_kfull(st), 64 * hh,
                        t * kBN, h, b);
        }
        __syncwarp();
      }
    }
    if (*abort_flag && lane == 0) {
      // Drain: let every copy this CTA started land before shared memory is released.
      for (int s2 = q_issued > 2 ? q_issued - 2 : 0; s2 < q_issued; ++s2)
        mbar_wait_quiet(bar_qfull(s2 & 1), (s2 >> 1) & 1);
      drain_ring<kStagesK>(bar_kfull0, kr);
    }
  } else if (warp == 2) {
    // ======================= V producer =======================
    const int nkv = p.n_ktiles;
    long long w, w_end;
    sk_range(p, &w, &w_end);
    if (lane == 0) tma_prefetch_desc(&p.tm_v);
    int vr = 0;
    bool ok = true;
    while (ok && w < w_end) {
      const SkSeg sg = sk_seg(w, w_end, nkv);
      w += sg.k1 - sg.k0;
      const int bh = sg.u / p.n_cta_m;
      const int h = bh % p.nh, b = bh / p.nh;
      for (int t = sg.k0; t < sg.k1; ++t, ++vr) {
        const int st = vr % kStagesV;
        const uint32_t ph = (vr / kStagesV) & 1;
        if (!warp_wait(bar_vempty(st), ph ^ 1, abort_flag, p.err)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(bar_vfull(st), C::kKVTileBytes);
#pragma unroll
          for (int hh = 0; hh < C::kHalves; ++hh)
            tma_load_4d(s_v0 + st * C::kKVTileBytes + hh * (kBN * 128), &p.tm_v, bar_vfull(st), 64 * hh,
                        t * kBN, h, b);
        }
        __syncwarp();
      }
    }
    if (*abort_flag && lane == 0) drain_ring<kStagesV>(bar_vfull0, vr);
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    // Per segment the issue order of flash2_fwd_kernel (S_0(j+1), P_1(j-1) V,
    // S_1(j+1), P_0(j) V); the next segment's first S follows the last P_0 V
    // and comes before the last P_1 V (tile 1 runs part of a step behind).
    constexpr uint32_t idesc_s = make_idesc_f16_f32(kBM, kBN, false);
    constexpr uint32_t idesc_pv = make_idesc_f16_f32(kBM, kD, true);
    const uint32_t tm = __shfl_sync(0xffffffffu, tmem, 0);
    const uint64_t dqa0 = make_sdesc_sw128(buf(0), 16, 1024);
    const uint64_t dqa1 = make_sdesc_sw128(buf(0) + kQTileBytes, 16, 1024);
    const uint64_t dqb0 = make_sdesc_sw128(buf(1), 16, 1024);
    const uint64_t dqb1 = make_sdesc_sw128(buf(1) + kQTileBytes, 16, 1024);
    const uint64_t dk0 = make_sdesc_sw128(s_k0, 16, 1024);
    const uint64_t dv0 = make_sdesc_sw128(s_v0, HD == 64 ? 8192 : kBN * 128, 1024);
    constexpr uint64_t kStageEnc = C::kKVTileBytes >> 4;
    constexpr uint64_t kQHalfEnc = (kBM * 128) >> 4;
    constexpr uint64_t kKHalfEnc = (kBN * 128) >> 4;
    auto issue_s = [&](int i, int st, int qb) {
      const uint64_t a = qb ? (i ? dqb1 : dqb0) : (i ? dqa1 : dqa0);
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
    // First S MMAs of segment seg_ (K ring position kr_, per-tile step
    // counts g0_ / g1_ before it).
    auto issue_first = [&](int seg_, int kr_, int g0_, int g1_, bool q1_) -> bool {
      const int qb = seg_ & 1;
      if (!warp_wait_issuer(bar_qfull(qb), (seg_ >> 1) & 1, abort_flag, p.err)) return false;
      if (!warp_wait_issuer(bar_kfull(kr_ % kStagesK), (kr_ / kStagesK) & 1, abort_flag, p.err)) return false;
      // S columns free: the softmax warps loaded the previous segment's last S.
      if (g0_ > 0 && !warp_wait_issuer(bar_sfree(0), (g0_ - 1) & 1, abort_flag, p.err)) return false;
      tc_fence_after();
      issue_s(0, kr_ % kStagesK, qb);
      if (q1_) {
        if (g1_ > 0 && !warp_wait_issuer(bar_sfree(1), (g1_ - 1) & 1, abort_flag, p.err)) return false;
        tc_fence_after();
        issue_s(1, kr_ % kStagesK, qb);
      }
      commit_to(bar_kempty(kr_ % kStagesK));
      return true;
    };

    const int nkv = p.n_ktiles;
    long long w, w_end;
    sk_range(p, &w, &w_end);
    // Ring positions and per-tile step counts run on across segments, so
    // every barrier parity continues where the previous segment left it.
    // Each round: the first S of segment `seg`, then the last P_1 V of the
    // segment before (still pending), then the rest of segment `seg` up to
    // its last P_0 V. (One call site of issue_first: a second inlined copy
    // makes this 64-register warp spill.)
    int kr = 0, vr = 0, g0 = 0, g1 = 0, seg = 0;
    bool ok = true;
    bool tail = false, tail_pv = false;  // pending: last P_1 V (if tile 1 ran) and its V release
    int tail_sv = 0, tail_j = 0, tail_par = 0;
    while (ok) {
      const bool has_seg = w < w_end;
      SkSeg sg = {0, 0, 0};
      int n = 0, n1 = 0;
      bool q1 = false;
      if (has_seg) {
        sg = sk_seg(w, w_end, nkv);
        q1 = 2 * (sg.u % p.n_cta_m) + 1 < p.n_qtiles;
        n = sg.k1 - sg.k0;
        n1 = q1 ? n : 0;
        if (SK_LOOKAHEAD && !issue_first(seg, kr, g0, g1, q1)) { ok = false; break; }
      }
      if (tail) {
        if (tail_pv) {
          if (!warp_wait_issuer(bar_p(1), tail_par, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          issue_pv(1, tail_sv, tail_j);
        }
        commit_to(bar_vempty(tail_sv));
        tail = false;
      }
      if (!has_seg) break;
      if (!SK_LOOKAHEAD && !issue_first(seg, kr, g0, g1, q1)) { ok = false; break; }
      const int qb = seg & 1;
      for (int j = 0; j < n; ++j) {
        const bool s_next = j + 1 < n;
        const int rk = kr + j + 1;
        const int sk = rk % kStagesK;
        if (s_next) {
          if (!warp_wait_issuer(bar_kfull(sk), (rk / kStagesK) & 1, abort_flag, p.err)) { ok = false; break; }
          if (!warp_wait_issuer(bar_sfree(0), (g0 + j) & 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, sk, qb);
        }
        if (j >= 1) {
          // P_1 V of the previous KV tile, then that V stage is free.
          const int sv = (vr + j - 1) % kStagesV;
          if (j - 1 < n1) {
            if (!warp_wait_issuer(bar_p(1), (g1 + j - 1) & 1, abort_flag, p.err)) { ok = false; break; }
            tc_fence_after();
            issue_pv(1, sv, j - 1);
          }
          commit_to(bar_vempty(sv));
        }
        if (s_next && j + 1 < n1) {
          if (!warp_wait_issuer(bar_sfree(1), (g1 + j) & 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          issue_s(1, sk, qb);
        }
        if (s_next) commit_to(bar_kempty(sk));
        const int rv0 = vr + j;
        const int sv = rv0 % kStagesV;
        if (!warp_wait_issuer(bar_vfull(sv), (rv0 / kStagesV) & 1, abort_flag, p.err)) { ok = false; break; }
        if (!warp_wait_issuer(bar_p(0), (g0 + j) & 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, sv, j);
      }
      tail = true;
      tail_pv = n1 > 0;
      tail_sv = (vr + n - 1) % kStagesV;
      tail_j = n - 1;
      tail_par = (g1 + n - 1) & 1;
      kr += n;
      vr += n;
      g0 += n;
      g1 += n1;
      ++seg;
      w += n;
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
    const int i = (warp - 4) >> 2;               // query tile of each unit: 0 or 1
    const int t = threadIdx.x - 128 * (1 + i);   // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t tS = tmem + lane_base + col_s(i);
    const uint32_t tP = tmem + lane_base + col_p(i);
    const uint32_t tO = tmem + lane_base + col_o(i);
    const int nkv = p.n_ktiles;
    long long w, w_end;
    sk_range(p, &w, &w_end);
    const float sc = p.scale_log2;
    const bool prescale = !(sc > 0.0f);  // negative scales: scale before max/mask
    bool ok = true;
    // Tile 1 starts part-way into tile 0's first KV step (see flash2_fwd_kernel).
    bool stagger_sent = (i != 0);
    bool stagger_seen = (i == 0);
    int gb = 0;      // KV steps this tile has run in earlier segments
    int pend_x = 0;  // buffer + 1 whose store read has not been waited for (thread t == 0)
    for (int seg = 0; ok && w < w_end; ++seg) {
      const SkSeg sg = sk_seg(w, w_end, nkv);
      w += sg.k1 - sg.k0;
      const int cta_m = sg.u % p.n_cta_m, bh = sg.u / p.n_cta_m;
      const int qb = seg & 1;
      if (i == 1 && 2 * cta_m + 1 >= p.n_qtiles) {
        // unit with one query tile: release this tile's share of the buffer
        __syncwarp();
        if (t == 0) mbar_arrive(bar_xfree(qb));
        continue;
      }
      const int n = sg.k1 - sg.k0;
      const int q_start = (2 * cta_m + i) * kBM;
      if (!stagger_seen) {
        ok = warp_wait(bar_stagger, 0, abort_flag, p.err);
        stagger_seen = true;
        if (!ok) break;
      }
      float m_ref = -INFINITY;
      float l = 0.0f;
      for (int j = 0; ok && j < n; ++j) {
        if (!warp_wait(bar_s(i), (gb + j) & 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[kBN];
        tmem_ld128_wait(tS, sr);
        // S_i is in registers: let the tensor core overwrite it with the next S.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sfree(i));
        float s[kBN];
#pragma unroll
        for (int c = 0; c < kBN; ++c) s[c] = __uint_as_float(sr[c]);
        float scl = sc;
        if (prescale) {
#pragma unroll
          for (int c = 0; c < kBN; ++c) s[c] *= sc;
          scl = 1.0f;
        }
        // keys visible to this row: c < nk - k_start (ragged last KV tile)
        const long long lim = p.nk - static_cast<long long>(sg.k0 + j) * kBN;
        if (lim < kBN) {
          const int limit = lim < 0 ? 0 : static_cast<int>(lim);
#pragma unroll
          for (int c = 0; c < kBN; ++c) s[c] = (c < limit) ? s[c] : -INFINITY;
        }
        float mxp, mxm;
        {
          constexpr int kNP = poly_cols(kBN), kNM = kBN - kNP;
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
        const float m_tile = mx * scl;
        const float m_new = fmaxf(m_ref, m_tile);
        const bool need = m_new > m_ref + kRescaleThreshold;
        float alpha = 1.0f;
        if (need) {
          alpha = ex2_approx(m_ref - m_new);
          m_ref = m_new;
        }
        l *= alpha;
        if (j > 0) {
          // P V of the previous step must be done before its P columns are
          // rewritten and before O is rescaled.
          if (!warp_wait(bar_pv(i), (gb + j - 1) & 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
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
        }
        const float m_use = (m_ref == -INFINITY) ? 0.0f : m_ref;
        const float2 scl2 = make_float2(scl, scl);
        const float2 nm2 = make_float2(-m_use, -m_use);
        float2 lsum[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int c = q * 32 + 2 * e;
            const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), scl2, nm2);
            const float2 pp = ((kPolyPairs >> (e & 7)) & 1)
                                  ? exp2_poly2(x)
                                  : make_float2(ex2_approx(x.x), ex2_approx(x.y));
            lsum[e & 3] = __fadd2_rn(lsum[e & 3], pp);
            pk[e] = pack_f16x2(pp.x, pp.y);
          }
          tmem_st16(tP + q * 16, pk);
          if (q == 2 && !stagger_sent) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_stagger);
            stagger_sent = true;
          }
        }
        {
          const float2 a = __fadd2_rn(lsum[0], lsum[1]);
          const float2 b = __fadd2_rn(lsum[2], lsum[3]);
          l += (a.x + a.y) + (b.x + b.y);
          // l sees the fp16 rounding of the tile's largest p (see flash2_fwd_kernel)
          const float xm = fmaf(mx, scl, -m_use);
          const float pm = (mxp >= mxm) ? exp2_poly2(make_float2(xm, xm)).x : ex2_approx(xm);
          l += __half2float(__float2half_rn(pm)) - pm;
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_p(i));
        if (SK_DEFER_READ && t == 0 && pend_x) {
          tma_store_wait_read0();
          mbar_arrive(bar_xfree(pend_x - 1));
          pend_x = 0;
        }
      }
      if (!stagger_sent) {
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_stagger);
        stagger_sent = true;
      }
      if (!ok) break;

      // ---- segment epilogue ----
      ok = warp_wait(bar_pv(i), (gb + n - 1) & 1, abort_flag, p.err);
      gb += n;
      if (!ok) break;
      tc_fence_after();
      uint32_t o[kD];
      {
        uint32_t tmp[32];
#pragma unroll
        for (int h = 0; h < kD / 32; ++h) {
          tmem_ld32_wait(tO + h * 32, tmp);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[32 * h + c] = tmp[c];
        }
      }
      float inv_l = (l > 0.0f) ? 1.0f / l : 0.0f;
      float lse2 = (l > 0.0f) ? m_ref + log2f(l) : -INFINITY;  // log2-sum-exp of the row
      bool store = true;
      if (!(sg.k0 == 0 && sg.k1 == nkv)) {
        // ---- a piece of a unit cut between consecutive CTAs ----
        const long long u0 = static_cast<long long>(sg.u) * nkv;
        const int c_first = sk_cta_of(p, u0);
        const int m = sk_cta_of(p, u0 + nkv - 1) - c_first + 1;
        const long long lse_off = static_cast<long long>(4 * p.sk_grid) * kD * kBM;
        // slot of piece pc: (its CTA, that CTA's first (0) or last (1) segment, tile)
        auto slot_of = [&](int pc) {
          const int c = c_first + pc;
          const int last_seg = (pc == 0 && p.sk_total * c / p.sk_grid != u0) ? 1 : 0;
          return static_cast<long long>((c * 2 + last_seg) * 2 + i);
        };
        const long long my = slot_of(static_cast<int>(blockIdx.x) - c_first);
        float4* so = reinterpret_cast<float4*>(p.sk_ws) + my * (kD / 4) * kBM;
#pragma unroll
        for (int c = 0; c < kD; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * inv_l);
#pragma unroll
        for (int c = 0; c < kD / 4; ++c)
          so[c * kBM + t] = make_float4(__uint_as_float(o[4 * c]), __uint_as_float(o[4 * c + 1]),
                                        __uint_as_float(o[4 * c + 2]), __uint_as_float(o[4 * c + 3]));
        p.sk_ws[lse_off + my * kBM + t] = lse2;
        // Release: the tile's stores, then (after the barrier) one fence by the
        // thread that counts the arrival (fences are cumulative).
        named_bar_sync(1 + i, 128);
        volatile unsigned* last_word = reinterpret_cast<volatile unsigned*>(smem + SC::kSmemFlag) + i;
        if (t == 0) {
          // Arrivals counted in the low byte, tagged with this launch's epoch
          // in the rest: a word an earlier launch left behind counts as zero.
          // At most m rounds: only this unit's m pieces touch the word.
          __threadfence();
          unsigned* cnt = p.sk_cnt + c_first * 2 + i;
          const unsigned ep = p.sk_epoch << 8;
          unsigned cur = *reinterpret_cast<volatile unsigned*>(cnt);
          unsigned nw;
          while (true) {
            nw = ((cur & ~0xffu) == ep) ? cur + 1u : (ep | 1u);
            const unsigned prev = atomicCAS(cnt, cur, nw);
            if (prev == cur) break;
            cur = prev;
          }
          const bool last = (nw & 0xffu) == static_cast<unsigned>(m);
          if (last) {
            *reinterpret_cast<volatile unsigned*>(cnt) = 0u;  // every piece has arrived
            __threadfence();  // acquire: the other pieces' stores are visible to the tile after the barrier
          }
          *last_word = last ? 1u : 0u;
        }
        named_bar_sync(1 + i, 128);
        store = *last_word != 0u;
        if (store) {
          // Merge every piece in piece order: O = sum_p 2^(lse_p - M) O_p / sum_p 2^(lse_p - M).
          float mx = -INFINITY;
          for (int pc = 0; pc < m; ++pc) mx = fmaxf(mx, __ldcg(p.sk_ws + lse_off + slot_of(pc) * kBM + t));
          // (o, already stored as this piece, becomes the accumulator)
#pragma unroll
          for (int c = 0; c < kD; ++c) o[c] = 0u;
          float wsum = 0.0f;
          for (int pc = 0; pc < m; ++pc) {
            const long long sl = slot_of(pc);
            const float lp = __ldcg(p.sk_ws + lse_off + sl * kBM + t);
            const float wp = (lp == -INFINITY) ? 0.0f : ex2_approx(lp - mx);
            wsum += wp;
            const float4* src = reinterpret_cast<const float4*>(p.sk_ws) + sl * (kD / 4) * kBM;
#pragma unroll
            for (int c = 0; c < kD / 4; ++c) {
              const float4 v = __ldcg(src + c * kBM + t);
              o[4 * c] = __float_as_uint(fmaf(wp, v.x, __uint_as_float(o[4 * c])));
              o[4 * c + 1] = __float_as_uint(fmaf(wp, v.y, __uint_as_float(o[4 * c + 1])));
              o[4 * c + 2] = __float_as_uint(fmaf(wp, v.z, __uint_as_float(o[4 * c + 2])));
              o[4 * c + 3] = __float_as_uint(fmaf(wp, v.w, __uint_as_float(o[4 * c + 3])));
            }
          }
          inv_l = wsum > 0.0f ? 1.0f / wsum : 0.0f;
          lse2 = wsum > 0.0f ? mx + log2f(wsum) : -INFINITY;
        }
      }
      if (store) {
        if (p.lse != nullptr && q_start + t < p.nq)
          p.lse[static_cast<long long>(bh) * p.nq + q_start + t] =
              (lse2 == -INFINITY) ? -INFINITY : lse2 * 0.69314718055994531f;
        // Stage the fp16 tile in this segment's buffer (its Q is no longer
        // read: every S MMA of the segment has completed) with the 128B
        // swizzle the TMA store expects.
        uint8_t* row = smem + (qb ? SC::kSmemBufB : C::kSmemQ) + i * kQTileBytes + t * 128;
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
        named_bar_sync(1 + i, 128);
        if (t == 0) {
          if (!*abort_flag) {
#pragma unroll
            for (int hh = 0; hh < C::kHalves; ++hh)
              tma_store_4d(&p.tm_o, buf(qb) + i * kQTileBytes + hh * (kBM * 128), 64 * hh, q_start, bh % p.nh,
                           bh / p.nh);
            tma_store_commit();
            if (!SK_DEFER_READ) tma_store_wait_read0();
          }
          if (SK_DEFER_READ) {
            pend_x = qb + 1;
          } else {
            mbar_arrive(bar_xfree(qb));  // the store has read the buffer
          }
        }
      } else {
        if (t == 0) mbar_arrive(bar_xfree(qb));
      }
    }
    if (!stagger_sent) {  // no segment, or stopped early
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_stagger);
    }
    if (t == 0) {
      tma_store_wait_read0();
      if (SK_DEFER_READ && pend_x) mbar_arrive(bar_xfree(pend_x - 1));
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
namespace {

// Workspace of one (device, stream): launches on a stream run in order, so
// one launch at a time uses it; launches on other streams have their own.
// Created on first use (never while its stream is being captured) and kept,
// for at most kMaxSkWorkspaces streams per device: a caller that makes a new
// stream per request must not grow device memory without bound, so further
// streams run the one-unit-per-CTA schedule.
constexpr int kMaxSkWorkspaces = 8;
struct SkWorkspace {
  float* ws = nullptr;
  unsigned* cnt = nullptr;
  size_t ws_floats = 0;
  size_t cnt_words = 0;
  unsigned epoch = 0;
};

std::mutex& sk_mutex() {
  static std::mutex mu;
  return mu;
}

std::map<std::pair<int, uintptr_t>, SkWorkspace>& sk_workspaces() {
  static std::map<std::pair<int, uintptr_t>, SkWorkspace> m;
  return m;
}

// FL_STREAMK: 0 never, 1 (default) where the cost model says it pays off,
// 2 whenever the shape allows it (tests).
int sk_mode() {
  static const int mode = [] {
    const char* e = std::getenv("FL_STREAMK");
    if (e == nullptr || *e == '\0') return 1;
    const int v = std::atoi(e);
    return (v < 0 || v > 2) ? 1 : v;
  }();
  return mode;
}

// Cost model in KV steps per SM, fitted to B200 measurements of both
// schedules (B1 H11, H14, H20, H23, H37 N4096, B4 H8 N4096, B1 H6 and H10
// N8192, B2 H8 N8192: 1.2 to 4 waves). One unit per CTA takes ceil(waves) *
// n_ktiles steps; stream-K 0.96 of its even share plus 0.375 * n_ktiles (the
// set-up, two segment changes with their merges, the SMs that finish late).
// Taken from a 1 % gain: BASELINE config 3 (1.73 waves, 65.1 against 64
// steps; measured 636 against 640 TF/s) keeps one unit per CTA, B1 H20 N4096
// (2.16 waves) gains 23 %.
bool sk_pays_off(long long units, int nkv, int sms) {
  if (units <= sms) return false;  // one wave or less: the split-KV launch covers it
  const double waves = static_cast<double>(units) / sms;
  const double t_units = std::ceil(waves) * nkv;
  const double t_sk = 0.96 * waves * nkv + 0.375 * nkv;
  return t_sk < 0.99 * t_units;
}

}  // namespace

cudaError_t launch_flash2_sk(Flash2Params prm, long long units, cudaStream_t stream, bool* launched) {
  *launched = false;
  const int mode = sk_mode();
  const int sms = sm_count();
  if (mode == 0 || units <= 0 || prm.n_ktiles <= 0) return cudaSuccess;
  if (mode == 1 && !sk_pays_off(units, prm.n_ktiles, sms)) return cudaSuccess;
  const long long total = units * prm.n_ktiles;
  const int grid = static_cast<int>(total < sms ? total : sms);  // every CTA gets a step
  const size_t ws_floats = static_cast<size_t>(4) * grid * (64 + 1) * kBM;
  const size_t cnt_words = static_cast<size_t>(2) * grid;
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(sk_mutex());
    auto& cache = sk_workspaces();
    const std::pair<int, uintptr_t> key{dev, reinterpret_cast<uintptr_t>(stream)};
    auto it = cache.find(key);
    if (it == cache.end() || it->second.ws == nullptr) {
      int on_dev = 0;  // workspaces that hold memory on this device
      for (const auto& kv : cache) on_dev += (kv.first.first == dev && kv.second.ws != nullptr) ? 1 : 0;
      if (on_dev >= kMaxSkWorkspaces) return cudaSuccess;  // the other schedule
    }
    SkWorkspace& w = cache[key];
    if (w.ws == nullptr || w.ws_floats < ws_floats || w.cnt_words < cnt_words) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
        (void)cudaGetLastError();  // not a launch failure: take the other schedule
        return cudaSuccess;
      }
      if (cs != cudaStreamCaptureStatusNone) return cudaSuccess;
      if (w.ws != nullptr) {
        // cudaFree waits for the device, so no launch still reads the old buffer
        e = cudaFree(w.ws);
        w = SkWorkspace{};
        if (e != cudaSuccess) return e;
      }
      void* mem = nullptr;
      e = cudaMalloc(&mem, (ws_floats + cnt_words) * sizeof(float));
      if (e != cudaSuccess) return e;
      w.ws = static_cast<float*>(mem);
      w.cnt = reinterpret_cast<unsigned*>(w.ws + ws_floats);
      w.ws_floats = ws_floats;
      w.cnt_words = cnt_words;
      e = cudaMemset(w.cnt, 0, cnt_words * sizeof(unsigned));
      if (e != cudaSuccess) return e;
    }
    w.epoch = (w.epoch + 1) & 0xffffffu;
    if (w.epoch == 0) w.epoch = 1;
    prm.sk_ws = w.ws;
    prm.sk_cnt = w.cnt;
    prm.sk_epoch = w.epoch;
  }
  prm.sk_total = total;
  prm.sk_grid = grid;
  constexpr int kSmemAlloc = SkCfg<64>::kSmemAlloc;
  auto kern = flash2_fwd_sk_kernel<64>;
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
  *launched = true;
  return cudaLaunchKernelEx(&cfg, kern, prm);
}

}  // namespace fl
