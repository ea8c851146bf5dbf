"""The bounded-wait failure path on a GPU, without a fault, trap or hang.

fl_selftest_bounded_wait runs the protocol every kernel of the library uses
on barriers that nothing arrives on: one warp's wait runs out after a short
limit and records the timeout, the other warp sees the CTA abort flag and
returns early. The host then reads FL_ERR_DEVICE_TIMEOUT through
fl_device_error(), and the same context still runs an attention call that
matches the CPU oracle. (The reference's only error path is CUDA_CHECK,
thebigblender/FlashLite csrc/includes/flash_attn.h:15-22.)"""
import ctypes

import pytest
import torch

from oracle import attention_oracle as orc

FL_OK, FL_ERR_DEVICE_TIMEOUT = 0, 6
LIMIT_NS = 1_000_000  # 1 ms


@pytest.mark.gpu
def test_wait_runs_out_is_reported_and_device_stays_usable(cuda, fl_lib):
    from flashlite_b200 import flash_attn_wmma as fa

    stream = torch.cuda.current_stream(cuda)
    sp = ctypes.c_void_p(stream.cuda_stream)
    flags = ctypes.c_uint32(0)
    fl_lib.fl_device_error(sp, ctypes.byref(flags))  # start from a clear error word
    out = torch.full((4,), -1, dtype=torch.int64, device=cuda)
    for _ in range(2):  # twice: the error word is cleared on read and set again
        assert fl_lib.fl_selftest_bounded_wait(LIMIT_NS, out.data_ptr(), sp) == FL_OK
        st = fl_lib.fl_device_error(sp, ctypes.byref(flags))
        assert st == FL_ERR_DEVICE_TIMEOUT and (flags.value & 1), (st, flags.value)
        ok0, t0, ok1, t1 = out.tolist()
        assert ok0 == 0 and ok1 == 0, "both waits must give up"
        assert LIMIT_NS <= t0 < 200 * LIMIT_NS, t0  # ran to its own limit, then gave up
        assert t1 < 500_000_000, t1  # left through the abort flag, far before its 2 s limit
        assert fl_lib.fl_device_error(sp, ctypes.byref(flags)) == FL_OK and flags.value == 0

    # the context is intact: an attention call still matches the oracle
    q, k, v = orc.make_qkv(1, 2, 512, 64, seed=11)
    ref = orc.attention_fp32(q, k, v, 0.125, True)
    got = fa.forward_flash2(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, True)
    mx, mean = orc.error_metrics(got, ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)
    assert fa.device_error() == 0
