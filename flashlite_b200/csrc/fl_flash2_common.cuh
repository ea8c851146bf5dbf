// Shared by the FlashAttention-2 forward kernels (fl_flash2.cu: one or two
// query tiles per CTA; fl_flash2_sk.cu: the stream-K schedule): tile shapes,
// the shared-memory and TMEM maps, the launch parameters, bounded warp waits
// and the TMA ring producers. Definitions other than the launch parameters
// sit in an anonymous namespace, so each translation unit that includes this
// header gets its own copy.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "fl_internal.h"
#include "fl_ptx.cuh"

namespace fl {

struct Flash2Params {
  // 4-D maps {D, rows, H, B} with box {64, tile rows, 1, 1}, SW128; the
  // strides give the [B,H,N,D] or [B,N,H,D] layout, the kernel's coordinates
  // are the same for both: (64 * half, row, h, b).
  CUtensorMap tm_q;  // {D, Nq, H, B} fp16, box rows 128
  CUtensorMap tm_k;  // {D, Nk, H, B}, box rows = KV tile
  CUtensorMap tm_v;  // {D, Nk, H, B}, box rows = KV tile
  CUtensorMap tm_o;  // {D, Nq, H, B}, box rows 128 (unused in merge mode)
  float* o_acc;      // merge mode: [BH, Nq, D] fp32
  float* lse;        // merge mode: [BH, Nq] fp32 (natural log)
  unsigned int* err; // device error word
  int nq, nk;        // query / key rows per slice
  int bh;            // number of (b,h) slices
  int nh;            // heads per batch entry: slice bh is (b, h) = (bh / nh, bh % nh)
  int n_qtiles;      // ceil(nq / 128)
  int n_ktiles;      // ceil(nk / 128)
  int tiles_per_cta; // 1 or 2 query tiles per CTA
  int n_cta_m;       // ceil(n_qtiles / tiles_per_cta)
  long long q_offset, kv_offset;  // global positions of row 0 (causal mask)
  float scale_log2;  // sm_scale * log2(e)
  int first;         // merge mode: overwrite instead of merge
  // stream-K schedule (fl_flash2_sk.cu) only
  long long sk_total;  // KV steps of all units
  int sk_grid;         // CTAs sharing them
  float* sk_ws;        // partial tiles of cut units: 4 * sk_grid slots of [D/4][128] float4, then their [128] lse
  unsigned* sk_cnt;    // arrival counts per cut unit and tile (2 * sk_grid)
  unsigned sk_epoch;   // launch tag of the arrival counts (24 bits, never 0)
};

// Stream-K launch of a non-causal head_dim-64 forward with two query tiles
// per unit (fl_flash2_sk.cu). Sets *launched to false, launching nothing,
// when the schedule would not beat one unit per CTA for this shape, when it
// is disabled (FL_STREAMK=0), or when its workspace for `stream` does not
// exist yet while the stream is being captured into a graph.
cudaError_t launch_flash2_sk(Flash2Params prm, long long units, cudaStream_t stream, bool* launched);

namespace {

constexpr int kBM = 128;       // query rows per tile (UMMA M)
constexpr int kThreads = 384;  // 3 warpgroups
// Tensor Memory columns (512 allocated: the CTA owns the whole SM's TMEM).
constexpr uint32_t kTmemCols = 512;

// Per-head-dimension shape. Every shared-memory tile is made of 64-column
// (128-byte) swizzle atoms: a D = 128 row is two atoms side by side, each
// half of a tile stored as its own [rows x 64] block, loaded and stored by
// its own TMA copy.
//   D = 64:  128-key KV tiles; TMEM S 2 x 128 | O 2 x 64  | P 2 x 64 columns.
//   D = 128:  64-key KV tiles (a K or V tile is still 16 KB and a KV step
//            the same tensor-core work as at D = 64, with half the
//            exponentials); TMEM S 2 x 64 | O 2 x 128 | P 2 x 32 columns.
template <int HD>
struct Cfg {
  static_assert(HD == 64 || HD == 128, "head dimension 64 or 128");
  static constexpr int kD = HD;
  static constexpr int kBN = HD == 64 ? 128 : 64;      // keys per KV tile (UMMA N of S)
  static constexpr int kHalves = HD / 64;              // 64-column atoms per row
  static constexpr int kStagesK = 4;                   // K ring depth
  static constexpr int kStagesV = 4;                   // V ring depth
  static constexpr int kQTileBytes = kBM * HD * 2;     // 16 / 32 KB
  static constexpr int kKVTileBytes = kBN * HD * 2;    // 16 KB
  // Shared-memory map (offsets from a 1024-byte aligned base).
  static constexpr int kSmemQ = 0;                                        // 2 tiles
  static constexpr int kSmemK = kSmemQ + 2 * kQTileBytes;                 // kStagesK tiles
  static constexpr int kSmemV = kSmemK + kStagesK * kKVTileBytes;         // kStagesV tiles
  static constexpr int kSmemBar = kSmemV + kStagesV * kKVTileBytes;       // mbarriers
  // q | k full/empty | v full/empty | s_full, s_free, p_full, pv_done (x2) | drain | stagger
  static constexpr int kNumBars = 1 + 2 * kStagesK + 2 * kStagesV + 4 * 2 + 2;
  static constexpr int kSmemMisc = kSmemBar + kNumBars * 8;  // tmem base, abort flag
  static constexpr int kSmemBytes = kSmemMisc + 16;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;       // alignment slack
  // Register split between warpgroup 0 (producers, MMA) and the two softmax
  // warpgroups; 128 * producer + 256 * softmax <= 384 * 168, the launch total.
#ifndef FL_D128_REGS_SOFTMAX
#define FL_D128_REGS_SOFTMAX 216
#endif
#ifndef FL_D128_REGS_PRODUCER
#define FL_D128_REGS_PRODUCER 56
#endif
  static constexpr int kRegsProducer = HD == 64 ? 64 : FL_D128_REGS_PRODUCER;
  static constexpr int kRegsSoftmax = HD == 64 ? 216 : FL_D128_REGS_SOFTMAX;
  static_assert(128 * kRegsProducer + 256 * kRegsSoftmax <= 384 * 168, "register split");
  // TMEM columns: S (fp32, kBN), O (fp32, kD), P (fp16 pairs, kBN / 2).
  __host__ __device__ static constexpr uint32_t col_s(int i) { return i ? kBN : 0u; }
  __host__ __device__ static constexpr uint32_t col_o(int i) { return 2 * kBN + (i ? kD : 0); }
  __host__ __device__ static constexpr uint32_t col_p(int i) { return 384u + (i ? kBN / 2 : 0); }
};
static_assert(Cfg<64>::col_o(1) + 64 <= 384 && Cfg<128>::col_o(1) + 128 <= 384, "O below P");
static_assert(Cfg<64>::kSmemAlloc <= 227 * 1024 && Cfg<128>::kSmemAlloc <= 227 * 1024, "smem");

// A row maximum may exceed the reference maximum by up to this much (log2
// units) before O and l are rescaled: p <= 2^8 stays exact enough in fp16.
constexpr float kRescaleThreshold = 8.0f;

// Bit e set: column pair e (mod 8) of every 16-column group is exponentiated
// on the FMA pipe (exp2_poly2) instead of the MUFU (2 of 8 pairs; with the
// two tiles staggered, 1/8 and 2/8 measure the same and 3/8 or more is slower).
#ifndef FL_POLY_PAIRS
#define FL_POLY_PAIRS 0x11
#endif
constexpr unsigned kPolyPairs = FL_POLY_PAIRS;
// FMA-pipe columns of a row of `cols` scores (pattern repeats every 16 columns).
__host__ __device__ constexpr int poly_cols(int cols) {
  return cols / 8 * __builtin_popcount(kPolyPairs & 0xffu);
}
static_assert(poly_cols(64) >= 8 && poly_cols(64) <= 56, "both exp methods must get columns");

// Maximum of N values in four independent chains of 3-input max.
template <int N>
__device__ __forceinline__ float max_chains4(const float* v) {
  static_assert(N % 4 == 0 && N >= 8, "N must be a multiple of 4, at least 8");
  constexpr int L = N / 4;
  float part[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float* w = v + g * L;
    float a = fmaxf(w[0], w[1]);
    int e = 2;
#pragma unroll
    for (; e + 1 < L; e += 2) a = fmax3(a, w[e], w[e + 1]);
    if (e < L) a = fmaxf(a, w[e]);
    part[g] = a;
  }
  return fmax3(fmaxf(part[0], part[1]), part[2], part[3]);
}


// Number of KV tiles (of kBN keys) a query tile starting at row q_start must visit.
template <int kBN>
__device__ __forceinline__ int kv_tiles_for(const Flash2Params& p, bool causal, int q_start) {
  if (!causal) return p.n_ktiles;
  // last visible key position for the tile's last row
  const long long last = p.q_offset + q_start + kBM - 1 - p.kv_offset;
  if (last < 0) return 0;
  const long long t = last / kBN + 1;
  return t < p.n_ktiles ? static_cast<int>(t) : p.n_ktiles;
}

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int* err) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err);
  return __all_sync(0xffffffffu, ok);
}

// Variant for the MMA-issuing warp (see mbar_wait_issuer).
__device__ __forceinline__ bool warp_wait_issuer(uint32_t bar, uint32_t parity,
                                                 volatile int* abort_flag, unsigned int* err) {
  const bool ok = mbar_wait_issuer(bar, parity, abort_flag, err);
  return __all_sync(0xffffffffu, ok);
}

// TMA producer of one ring (K or V): tile t goes to stage t % kStages once
// the consumer released that stage (one copy per 64-column half). Returns
// the number of tiles issued.
template <int HD, int kStages>
__device__ __forceinline__ int produce_ring(const CUtensorMap* tm, uint32_t s_ring, uint32_t bar_full0,
                                            uint32_t bar_empty0, int n_tiles, int h, int b, int lane,
                                            volatile int* abort_flag, unsigned int* err) {
  using C = Cfg<HD>;
  int issued = 0;
  for (int t = 0; t < n_tiles; ++t) {
    const int st = t % kStages;
    const uint32_t ph = (t / kStages) & 1;
    if (!warp_wait(bar_empty0 + 8u * st, ph ^ 1, abort_flag, err)) break;
    if (lane == 0) {
      mbar_arrive_expect_tx(bar_full0 + 8u * st, C::kKVTileBytes);
#pragma unroll
      for (int hh = 0; hh < C::kHalves; ++hh)
        tma_load_4d(s_ring + st * C::kKVTileBytes + hh * (C::kBN * 128), tm, bar_full0 + 8u * st,
                    64 * hh, t * C::kBN, h, b);
    }
    __syncwarp();
    issued = t + 1;
  }
  return issued;
}

// Split-KV variant: slot 0 streams KV tiles [0, nkv0) and slot 1 tiles
// [kvb1, kvb1 + nkv1) of the same query tile; both sequences share one ring,
// interleaved (slot 0's step j, then slot 1's step j), so ring index 2j + i.
template <int HD, int kStages>
__device__ __forceinline__ int produce_ring_split(const CUtensorMap* tm, uint32_t s_ring, uint32_t bar_full0,
                                                  uint32_t bar_empty0, int nkv0, int nkv1, int kvb1, int h,
                                                  int b, int lane, volatile int* abort_flag, unsigned int* err) {
  using C = Cfg<HD>;
  int issued = 0;
  for (int j = 0; j < nkv0; ++j) {
    for (int i = 0; i < 2; ++i) {
      if (i == 1 && j >= nkv1) break;
      const int t = issued;
      const int st = t % kStages;
      const uint32_t ph = (t / kStages) & 1;
      if (!warp_wait(bar_empty0 + 8u * st, ph ^ 1, abort_flag, err)) return issued;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_full0 + 8u * st, C::kKVTileBytes);
#pragma unroll
        for (int hh = 0; hh < C::kHalves; ++hh)
          tma_load_4d(s_ring + st * C::kKVTileBytes + hh * (C::kBN * 128), tm, bar_full0 + 8u * st,
                      64 * hh, (j + (i ? kvb1 : 0)) * C::kBN, h, b);
      }
      __syncwarp();
      issued = t + 1;
    }
  }
  return issued;
}

template <int kStages>
__device__ __forceinline__ void drain_ring(uint32_t bar_full0, int issued) {
  for (int t = issued > kStages ? issued - kStages : 0; t < issued; ++t)
    mbar_wait_quiet(bar_full0 + 8u * (t % kStages), (t / kStages) & 1);
}

}  // namespace
}  // namespace fl
