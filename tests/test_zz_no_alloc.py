"""GPU test of the allocation-free block step (fl_flash2_fwd_block_noalloc).

That entry point exists for callers that cannot allocate device memory when
they call the library (a host runtime that owns all device memory after
start-up, or a latency-critical path where an allocation may stall or fail):
its running attention state lives in a fixed array inside the library.

Checks, through the C ABI: two calls in a row, each against the existing
entry point (fl_flash2_fwd_block with caller buffers + fl_ring_finalize) on
the same inputs; a multi-block first..last sequence; no device memory is
allocated by a call; sizes beyond the array's 65536 rows are rejected.
Collected last on purpose (file name), and independent of test order.
"""
import ctypes
import gc

import pytest
import torch

from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

P, I64, F32, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
FL_ERR_UNSUPPORTED = 2


@pytest.fixture(scope="module")
def lib(fl_lib):
    fl_lib.fl_flash2_fwd_block_noalloc.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, I64, F32,
                                                   I32, I32, I32, P]
    fl_lib.fl_flash2_fwd_block_noalloc.restype = I32
    return fl_lib


def _existing(lib, q, k, v, q_off, kv_off, causal, first, o_acc, lse):
    BH, Nq, Nk = q.shape[0] * q.shape[1], q.shape[2], k.shape[2]
    st = lib.fl_flash2_fwd_block(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_acc.data_ptr(),
                                 lse.data_ptr(), BH, Nq, Nk, 64, q_off, kv_off, 0.125,
                                 int(causal), int(first), None)
    assert st == 0, lib.fl_last_error()


def _noalloc(lib, q, k, v, o, q_off, kv_off, causal, first, last):
    BH, Nq, Nk = q.shape[0] * q.shape[1], q.shape[2], k.shape[2]
    st = lib.fl_flash2_fwd_block_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                         o.data_ptr() if o is not None else None, BH, Nq, Nk, 64,
                                         q_off, kv_off, 0.125, int(causal), int(first), int(last),
                                         None)
    assert st == 0, lib.fl_last_error()


def _reference_single(lib, q, k, v, q_off, kv_off, causal):
    o_acc = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    _existing(lib, q, k, v, q_off, kv_off, causal, True, o_acc, lse)
    out = torch.empty_like(q)
    assert lib.fl_ring_finalize(o_acc.data_ptr(), out.data_ptr(), out.numel(), None) == 0
    return out


def _close(a, b):
    mx, mean = orc.error_metrics(a, b)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)


def test_two_calls_in_a_row_match_existing_entry_point(cuda, lib):
    # call 1: a larger block; call 2: a smaller one, so stale state from call 1
    # sits in the shared array beyond call 2's rows
    cases = [((2, 4, 512), (2, 4, 640), 640, 0, True), ((1, 3, 200), (1, 3, 300), 0, 0, False)]
    for (qs, ks, q_off, kv_off, causal) in cases:
        q, _, _ = (t.to(cuda) for t in orc.make_qkv(*qs, 64, seed=qs[2]))
        _, k, v = (t.to(cuda) for t in orc.make_qkv(*ks, 64, seed=ks[2] + 1))
        o = torch.full_like(q, float("nan"))
        _noalloc(lib, q, k, v, o, q_off, kv_off, causal, True, True)
        ref = _reference_single(lib, q, k, v, q_off, kv_off, causal)
        torch.cuda.synchronize()
        assert not torch.isnan(o.float()).any()
        _close(o.cpu(), ref.cpu())


def test_multi_block_sequence_matches_full_attention(cuda, lib):
    nb, H, P = 256, 4, 3
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, H, nb * P, 64, seed=77))
    full = orc.attention_fp32(q.cpu(), k.cpu(), v.cpu(), 0.125, True)
    r = P - 1  # the last block sees every key block
    qb = q[:, :, r * nb:].contiguous()
    o = torch.empty_like(qb)
    for s in range(P):
        src = r - s
        kb = k[:, :, src * nb:(src + 1) * nb].contiguous()
        vb = v[:, :, src * nb:(src + 1) * nb].contiguous()
        _noalloc(lib, qb, kb, vb, o if s == P - 1 else None, r * nb, src * nb, True,
                 s == 0, s == P - 1)
    torch.cuda.synchronize()
    _close(o.cpu(), full[:, :, r * nb:])


def test_call_allocates_no_device_memory(cuda, lib):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, 2, 256, 64, seed=5))
    o = torch.empty_like(q)
    # The first call on the device does the set-up (symbol lookup) and, being
    # the same launch as the loop below, also loads every kernel the loop
    # uses, so nothing lazily loaded can show up as device memory later.
    _noalloc(lib, q, k, v, o, 0, 0, True, True, True)
    torch.cuda.synchronize()
    gc.collect()  # tensors of earlier tests still waiting for collection
    free0, _ = torch.cuda.mem_get_info()
    torch_alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        _noalloc(lib, q, k, v, o, 0, 0, True, True, True)
    torch.cuda.synchronize()
    # torch may free (never allocate) blocks of earlier tests meanwhile
    assert torch.cuda.memory_allocated() <= torch_alloc0
    # Device-wide free memory also counts other contexts on the GPU, so it is
    # compared with slack: an allocation by these calls would be at least the
    # 2 MiB allocation granule.
    assert torch.cuda.mem_get_info()[0] >= free0 - (1 << 20)


def test_rejects_sizes_beyond_the_array(cuda, lib):
    buf = torch.zeros(64, dtype=torch.float16, device=cuda)
    p = buf.data_ptr()
    st = lib.fl_flash2_fwd_block_noalloc(p, p, p, p, 2, 32769, 128, 64, 0, 0, 0.125, 1, 1, 1, None)
    assert st == FL_ERR_UNSUPPORTED
    assert b"65536" in lib.fl_last_error()
