/*
 * flashlite_b200 — C ABI of the B200 (sm_100a) FlashAttention-2 forward engine.
 *
 * Plain pointers and sizes only: no torch, no C++ types. Every tensor is a
 * contiguous fp16 array laid out [B, H, N, D] (element (b,h,n,d) at offset
 * ((b*H + h)*N + n)*D + d), resident in device memory of the current device.
 * Calls are asynchronous on `stream` (a cudaStream_t passed as void*; NULL =
 * the legacy default stream) and return a status code; a non-zero status
 * means nothing was launched. Errors found by a kernel while it runs (a
 * bounded wait that gave up) are reported by fl_device_error().
 *
 * Reference interface being replaced (thebigblender/FlashLite):
 *   csrc/includes/flash_attn.h:100-124   host declarations
 *   csrc/flash_attn.cpp:4-29             pybind11 module `flash_attn_wmma`
 */
#ifndef FLASHLITE_B200_H_
#define FLASHLITE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
typedef enum fl_status {
  FL_OK = 0,
  FL_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, size overflow      */
  FL_ERR_UNSUPPORTED = 2,      /* e.g. head_dim != 64 for the FA2 kernel       */
  FL_ERR_MISALIGNED = 3,       /* a pointer is not 16-byte aligned             */
  FL_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed            */
  FL_ERR_NO_DEVICE = 5,        /* current device is not sm_100 (B200 class)    */
  FL_ERR_DEVICE_TIMEOUT = 6    /* a kernel's bounded wait gave up (see below)  */
} fl_status;

/*
 * FlashAttention-2 forward: o = softmax(q k^T * sm_scale [causal]) v.
 * Replaces flash_attn::flash_attn_forward_flash2 (csrc/kernel_flash2.cu:732-839).
 * q, k, v, o: [B, H, N, D] fp16, D must be 64 (csrc/kernel_flash2.cu:756-757).
 * sm_scale == 0 selects 1/sqrt(D) (csrc/kernel_flash2.cu:769-771).
 * is_causal != 0 masks keys j > query i. o may not alias q, k or v.
 * Device memory: a non-causal call whose grid would leave part of its last
 * wave idle may run the stream-K schedule; the first such call on a stream
 * allocates that stream's 19.7 MB workspace (cudaMalloc, kept until exit;
 * never while the stream is being captured: the call then runs the other
 * schedule). At most 8 streams per device get one; calls on further streams
 * run the other schedule. FL_STREAMK=0 in the environment turns the schedule
 * off. The same holds for fl_flash2_fwd_ex.
 */
int fl_flash2_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
                  int64_t N, int64_t D, float sm_scale, int is_causal, void* stream);

/* Tensor layouts accepted by fl_flash2_fwd_ex and fl_flash2_bwd. */
enum fl_layout {
  FL_LAYOUT_BHND = 0, /* [B, H, N, D]: the reference's layout */
  FL_LAYOUT_BNHD = 1  /* [B, N, H, D]: the flash_attn package's layout */
};

/*
 * FA2 forward with separate query / key lengths, global positions, an
 * optional log-sum-exp output and a choice of layout; no reference
 * counterpart (the reference's forward_flash2 assumes N_k == N_q without
 * checking it, csrc/kernel_flash2.cu:749-755, and takes [B, H, N, D] only).
 * q, o: [B, H, Nq, D] (or [B, Nq, H, D] with FL_LAYOUT_BNHD) fp16; k, v:
 * [B, H, Nk, D] (or [B, Nk, H, D]) fp16; D is 64 or 128 (the reference
 * takes 64 only, csrc/kernel_flash2.cu:756-757). Query row i sits at
 * position q_offset + i and key row j at kv_offset + j; with is_causal a
 * query sees the keys at positions <= its own. lse (may be NULL): [B, H, Nq]
 * fp32 in either layout, natural-log log-sum-exp of the scaled scores of
 * each row (-inf for a row without visible keys, whose output is zero).
 * sm_scale == 0 means 1/sqrt(D).
 */
int fl_flash2_fwd_ex(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                     int64_t H, int64_t Nq, int64_t Nk, int64_t D, int64_t q_offset,
                     int64_t kv_offset, float sm_scale, int is_causal, int layout, void* stream);

/*
 * FA2 backward; no reference counterpart (the reference is forward-only).
 * q, k, v, o, dout, dq, dk, dv: [B, H, N, 64] fp16, or [B, N, H, 64] with
 * layout FL_LAYOUT_BNHD (o = the forward output, dout = dL/do); lse:
 * [B, H, N] fp32 in either layout, the natural-log log-sum-exp the
 * forward returns (fl_flash2_fwd_ex with a non-NULL lse). Computes dq, dk,
 * dv of softmax(sm_scale * q k^T [causal mask]) v; sm_scale == 0 means
 * 1/sqrt(64). workspace: device memory of at least
 * fl_flash2_bwd_workspace_size(B, H, N, D) bytes, 16-byte aligned (fp32 dq
 * accumulator and per-row vectors; nothing is allocated by the call).
 */
size_t fl_flash2_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D);
int fl_flash2_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, void* workspace,
                  size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D,
                  float sm_scale, int is_causal, int layout, void* stream);

/*
 * Naive (unfused, fp32 CUDA-core) attention forward, any D in [1, 1024].
 * Replaces flash_attn::flash_attn_forward_naive (csrc/kernel_naive.cu:242-323).
 */
int fl_naive_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
                 int64_t N, int64_t D, float sm_scale, int is_causal, void* stream);

/*
 * One block step of sequence-sharded (ring) attention; no reference
 * counterpart (the reference is single-GPU). Attends the query block q
 * [BH, Nq, D] (global positions q_offset..q_offset+Nq-1, D = 64 or 128) to
 * the key/value block k, v [BH, Nk, D] (positions kv_offset..), causal by
 * global position when is_causal != 0, and merges the result into the
 * running state:
 *   o_acc  [BH, Nq, D]  fp32, normalised partial output
 *   lse    [BH, Nq]     fp32, natural-log sum-exp of the scaled scores
 * If `first` != 0 the running state is overwritten instead of merged.
 * Rows with no visible key keep (o_acc, lse) = (0, -inf) when `first`.
 */
int fl_flash2_fwd_block(const void* q, const void* k, const void* v, float* o_acc, float* lse,
                        int64_t BH, int64_t Nq, int64_t Nk, int64_t D, int64_t q_offset,
                        int64_t kv_offset, float sm_scale, int is_causal, int first,
                        void* stream);

/*
 * Final step of ring attention: o[i] = fp16(o_acc[i]) for BH*Nq*D elements.
 * No reference counterpart.
 */
int fl_ring_finalize(const float* o_acc, void* o, int64_t n_elems, void* stream);

/*
 * Allocation-free block step. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory when they call this library:
 * a host runtime that owns all device memory and hands out nothing after
 * start-up, or a latency-critical path where an allocation could stall or
 * fail. Same computation as fl_flash2_fwd_block, but the running state
 * (normalised fp32 output and log-sum-exp of B*H*Nq rows) lives in a fixed
 * 16.25 MiB array inside the library instead of caller buffers; nothing is
 * allocated. `first` != 0 starts a new accumulation (it overwrites the
 * state); `last` != 0 also writes the fp16 result to o [BH, Nq, 64] (o may
 * be NULL otherwise). Limits: D == 64 and BH*Nq <= 65536 rows, else
 * FL_ERR_UNSUPPORTED. Every GPU that loads the library holds the array until
 * the process exits. All calls on a device share that one array and it keeps
 * the last call's contents: a first..last sequence must not be interleaved
 * with another one, and calls that overlap on the GPU (other streams or
 * threads) race. The first call on each device looks up the array's device
 * address; make that first call before any stream capture begins.
 */
int fl_flash2_fwd_block_noalloc(const void* q, const void* k, const void* v, void* o,
                                int64_t BH, int64_t Nq, int64_t Nk, int64_t D, int64_t q_offset,
                                int64_t kv_offset, float sm_scale, int is_causal, int first,
                                int last, void* stream);

/* Human-readable text for a status code (static storage). */
const char* fl_status_str(int status);

/* Text of the last error raised on the calling thread ("" if none). */
const char* fl_last_error(void);

/*
 * Reads and clears the device error word of the current device after
 * synchronising `stream`. Writes the raw bit flags to *flags (may be NULL)
 * and returns FL_ERR_DEVICE_TIMEOUT if any kernel gave up a wait, else FL_OK.
 */
int fl_device_error(void* stream, uint32_t* flags);

/*
 * Self-test of the bounded-wait failure path. No reference counterpart: the
 * reference's only error path is CUDA_CHECK after a launch
 * (csrc/includes/flash_attn.h:15-22). Every wait inside this library's
 * kernels is bounded; this entry point makes one run out on purpose, in the
 * form a kernel can survive: one CTA of two warps on `stream`, each waiting
 * on its own mbarrier that nothing ever arrives on. Warp 0 waits at most
 * `limit_ns` (1 .. 1e9 ns), then records the timeout in the device error word
 * and raises its CTA's abort flag; warp 1 waits with the library's normal
 * limit (2 s) but sees the abort flag and returns early, as every role of the
 * attention kernels does. `out` (device memory, 4 x uint64) receives warp 0's
 * wait result (1 = completed, 0 = gave up), its wait time in ns, then the same
 * two values of warp 1. Afterwards fl_device_error() returns
 * FL_ERR_DEVICE_TIMEOUT and the device stays usable.
 */
int fl_selftest_bounded_wait(uint64_t limit_ns, uint64_t* out, void* stream);

/* Library version as "major.minor.patch". */
const char* fl_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FLASHLITE_B200_H_ */
