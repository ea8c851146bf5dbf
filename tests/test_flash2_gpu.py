"""GPU parity of the tcgen05 FA2 forward against the CPU fp32 oracle.

Tolerance (north star): max-abs <= 2e-3 and mean-abs <= 2e-4 against fp32
softmax(QK^T*scale)V on the same seeded fp16 inputs. Cases: the reference's
own test matrix (thebigblender/FlashLite tests/test_correctness.py:61-90),
the BASELINE configs 1-3, both dispatch classes (two query tiles per CTA, or
one query tile whose KV range is split between the CTA's two softmax
warpgroups), ragged N, N smaller than a tile, the default and a negative scale, the
zero-allocation ``out=`` form, and calls straight through the C ABI.
"""
import ctypes
import math

import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

TOL_MAX, TOL_MEAN = orc.MAX_ABS_TOL, orc.MEAN_ABS_TOL


def _check(out, ref, tag=""):
    mx, mean = orc.error_metrics(out, ref)
    assert out.dtype == torch.float16
    assert not torch.isnan(out.float()).any(), f"NaN in output {tag}"
    assert mx <= TOL_MAX and mean <= TOL_MEAN, f"{tag}: max-abs {mx:.3e} mean-abs {mean:.3e}"
    return mx, mean


def _run(cuda, B, H, N, causal, seed=0, sm_scale=0.125, input_scale=1.0):
    q, k, v = orc.make_qkv(B, H, N, 64, seed=seed, scale=input_scale)
    ref = orc.attention_fp32(q, k, v, sm_scale, causal)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    out = fa.forward_flash2(qd, kd, vd, sm_scale, causal)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    return _check(out.cpu(), ref, f"B{B} H{H} N{N} causal={causal}")


@pytest.mark.parametrize("batch_size", [1, 2])
@pytest.mark.parametrize("num_heads", [4, 8])
@pytest.mark.parametrize("seq_len", [128, 256, 512])
@pytest.mark.parametrize("is_causal", [False, True])
def test_reference_matrix(cuda, batch_size, num_heads, seq_len, is_causal):
    _run(cuda, batch_size, num_heads, seq_len, is_causal, seed=42, sm_scale=1.0 / math.sqrt(64))


@pytest.mark.parametrize("cfg", [
    (1, 2, 128, False),    # config 1
    (2, 8, 1024, False),   # config 2
    (2, 8, 1024, True),
    (2, 8, 4096, False),   # config 3 (headline)
    (2, 8, 4096, True),
], ids=lambda c: f"B{c[0]}H{c[1]}N{c[2]}{'c' if c[3] else ''}")
def test_baseline_configs(cuda, cfg):
    B, H, N, causal = cfg
    _run(cuda, B, H, N, causal, seed=0)


@pytest.mark.parametrize("N", [1, 37, 64, 100, 129, 200, 383, 1000, 1100, 2049])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_lengths(cuda, N, causal):
    _run(cuda, 1, 3, N, causal, seed=N)


@pytest.mark.parametrize("N,causal", [(1100, False), (1100, True), (2000, True), (640, False)])
def test_two_tiles_per_cta_dispatch(cuda, N, causal):
    # B*H large enough that two query tiles per CTA still fill 148 SMs,
    # with an odd number of query tiles for N = 1100 / 2000 / 640.
    _run(cuda, 4, 16, N, causal, seed=5)


@pytest.mark.parametrize("N", [384, 640, 1000, 2049])
@pytest.mark.parametrize("causal", [False, True])
def test_split_kv_one_tile_per_cta(cuda, N, causal):
    # Few (b,h) slices, so one query tile per CTA: its KV tiles are split
    # between the two softmax warpgroups (odd and even tile counts, ragged
    # keys, causal tiles whose second half is empty) and merged in the
    # epilogue; repeated calls give the same bits.
    q, k, v = orc.make_qkv(1, 2, N, 64, seed=N + 7)
    ref = orc.attention_fp32(q, k, v, 0.125, causal)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    a = fa.forward_flash2(qd, kd, vd, 0.125, causal)
    b = fa.forward_flash2(qd, kd, vd, 0.125, causal)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    assert torch.equal(a, b)
    _check(a.cpu(), ref, f"split N{N} causal={causal}")


@pytest.mark.parametrize("B,H,N,causal", [
    (1, 150, 200, False),   # 2 KV steps per CTA
    (1, 150, 200, True),
    (1, 160, 384, False),   # 3 query tiles: the second pair has one tile
    (1, 160, 384, True),
    (3, 50, 1000, True),    # causal pairs of 2..8 KV steps, ragged last tile
])
def test_many_two_tile_ctas(cuda, B, H, N, causal):
    # >= 148 two-tile CTAs (more than one wave), short and odd-length cases
    _run(cuda, B, H, N, causal, seed=B * H + N)


@pytest.mark.parametrize("B,H,N", [(2, 80, 1000), (1, 150, 256), (1, 148, 2048)])
def test_full_pairs_many_ctas_repeatable(cuda, B, H, N):
    # Non-causal, even query-tile count, >= 148 tile pairs (ragged keys and
    # rows for N = 1000), run twice: the bits repeat.
    q, k, v = orc.make_qkv(B, H, N, 64, seed=N + H)
    ref = orc.attention_fp32(q, k, v, 0.125, False)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    a = fa.forward_flash2(qd, kd, vd, 0.125, False)
    b = fa.forward_flash2(qd, kd, vd, 0.125, False)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    assert torch.equal(a, b)
    _check(a.cpu(), ref, f"B{B} H{H} N{N}")


@pytest.mark.parametrize("causal", [False, True])
def test_repeatable_two_tile_dispatch(cuda, causal):
    q, k, v = orc.make_qkv(4, 16, 1100, 64, seed=10)
    ref = orc.attention_fp32(q, k, v, 0.125, causal)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    first = fa.forward_flash2(qd, kd, vd, 0.125, causal)
    for _ in range(3):
        again = fa.forward_flash2(qd, kd, vd, 0.125, causal)
        assert torch.equal(first, again)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    _check(first.cpu(), ref, "repeat")


def test_default_and_negative_scale(cuda):
    _run(cuda, 1, 2, 256, False, seed=1, sm_scale=0.0)
    _run(cuda, 1, 2, 256, True, seed=2, sm_scale=-0.125)


def test_large_logits_rescale_path(cuda):
    # sm_scale 1.0 -> log2-domain logits with std ~11.5: the running maximum
    # grows by more than 2^8 often, exercising the conditional O rescale
    _run(cuda, 1, 4, 1024, False, seed=3, sm_scale=1.0)
    _run(cuda, 1, 4, 1024, True, seed=4, sm_scale=1.0)
    # the same over >= 148 full tile pairs (persistent launch: units split
    # between CTAs are merged from parts with different row maxima); inputs
    # scaled so |O| < 4, where one fp16 ulp of the output stays below the
    # absolute tolerance
    _run(cuda, 1, 150, 512, False, seed=5, sm_scale=2.0, input_scale=0.7)


@pytest.mark.parametrize("causal", [False, True])
def test_as_accurate_as_reference_numerics(cuda, causal):
    """Inputs x3 (|O| up to ~15, where fp16 output rounding alone exceeds
    2e-3): the error must stay within that of the reference kernel's own
    tiled numerics (oracle.flash2_tiled_reference) on the same inputs."""
    q, k, v = orc.make_qkv(1, 2, 512, 64, seed=6, scale=3.0)
    ref = orc.attention_fp32(q, k, v, 0.125, causal)
    ref_tiled = torch.from_numpy(orc.flash2_tiled_reference(q, k, v, 0.125, causal))
    mx_ref, mean_ref = orc.error_metrics(ref_tiled, ref)
    out = fa.forward_flash2(q.cuda(), k.cuda(), v.cuda(), 0.125, causal).cpu()
    mx, mean = orc.error_metrics(out, ref)
    assert mx <= 1.5 * mx_ref + 1e-3 and mean <= 1.5 * mean_ref + 1e-4, (mx, mean, mx_ref, mean_ref)


def test_out_buffer_zero_alloc(cuda):
    q, k, v = orc.make_qkv(2, 4, 512, 64, seed=8)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    out_buf = torch.empty_like(qd)
    fa.forward_flash2(qd, kd, vd, 0.125, True, out=out_buf)  # warm-up
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    res = fa.forward_flash2(qd, kd, vd, 0.125, True, out=out_buf)
    torch.cuda.synchronize()
    assert res.data_ptr() == out_buf.data_ptr()
    assert torch.cuda.memory_allocated() == before
    _check(out_buf.cpu(), orc.attention_fp32(q, k, v, 0.125, True), "out=")


@pytest.mark.parametrize("B,H,N,causal", [(2, 8, 1024, False), (2, 8, 4096, True), (1, 2, 640, False)])
def test_back_to_back_calls_see_previous_output(cuda, B, H, N, causal):
    # Each launch lets the next kernel on the stream start its set-up early;
    # a call that reads the previous call's output, issued without a
    # synchronisation in between, must still see all of it.
    q, k, v = orc.make_qkv(B, H, N, 64, seed=N + B)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    o1 = fa.forward_flash2(qd, kd, vd, 0.125, causal)
    o2 = fa.forward_flash2(o1, kd, vd, 0.125, causal)      # reads o1
    o3 = fa.forward_flash2(qd, o2, vd, 0.125, causal)      # reads o2 as keys
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    r1 = fa.forward_flash2(qd, kd, vd, 0.125, causal)
    torch.cuda.synchronize()
    r2 = fa.forward_flash2(r1, kd, vd, 0.125, causal)
    torch.cuda.synchronize()
    r3 = fa.forward_flash2(qd, r2, vd, 0.125, causal)
    torch.cuda.synchronize()
    assert torch.equal(o1, r1) and torch.equal(o2, r2) and torch.equal(o3, r3)
    if N <= 1024:
        ref2 = orc.attention_fp32(o1.cpu(), k, v, 0.125, causal)
        _check(o2.cpu(), ref2, "chained")


def test_deterministic(cuda):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(2, 8, 1024, 64, seed=9))
    a = fa.forward_flash2(q, k, v, 0.125, False)
    b = fa.forward_flash2(q, k, v, 0.125, False)
    assert torch.equal(a, b)


def test_binding_errors_on_gpu(cuda):
    q = torch.zeros(1, 2, 128, 64, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError, match="requires head_dim == 64"):
        z = torch.zeros(1, 2, 128, 32, dtype=torch.float16, device=cuda)
        fa.forward_flash2(z, z, z)
    with pytest.raises(RuntimeError, match="All tensors must be FP16"):
        fa.forward_flash2(q.float(), q.float(), q.float())
    with pytest.raises(RuntimeError, match="out tensor shape must match q"):
        fa.forward_flash2(q, q, q, out=torch.empty(1, 2, 64, 64, dtype=torch.float16, device=cuda))
    with pytest.raises(RuntimeError, match="All tensors must be contiguous"):
        t = torch.zeros(1, 128, 2, 64, dtype=torch.float16, device=cuda).transpose(1, 2)
        fa.forward_flash2(t, t, t)
    empty = torch.zeros(1, 2, 0, 64, dtype=torch.float16, device=cuda)
    assert fa.forward_flash2(empty, empty, empty).shape == empty.shape


def test_c_abi_direct(cuda, fl_lib):
    """The C entry point alone (no torch binding) on a raw stream."""
    B, H, N = 2, 4, 777
    q, k, v = orc.make_qkv(B, H, N, 64, seed=21)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    o = torch.empty_like(qd)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        st = fl_lib.fl_flash2_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(),
                                  B, H, N, 64, 0.0, 1, ctypes.c_void_p(stream.cuda_stream))
    assert st == 0, fl_lib.fl_last_error()
    flags = ctypes.c_uint32(99)
    assert fl_lib.fl_device_error(ctypes.c_void_p(stream.cuda_stream), ctypes.byref(flags)) == 0
    assert flags.value == 0
    _check(o.cpu(), orc.attention_fp32(q, k, v, 0.0, True), "C ABI")


def test_c_abi_misaligned(cuda, fl_lib):
    buf = torch.zeros(2 * 128 * 64 + 8, dtype=torch.float16, device=cuda)
    p = buf.data_ptr() + 2  # 2-byte offset
    assert fl_lib.fl_flash2_fwd(p, p, p, p, 1, 1, 128, 64, 0.0, 0, None) == 3


def test_head_sharded_slices_match_full(cuda):
    """Config-4 style sharding: each contiguous range of (b,h) slices run on
    its own gives the same bytes as the full call (no communication)."""
    B, H, N = 4, 8, 1024
    q, k, v = (t.to(cuda) for t in orc.make_qkv(B, H, N, 64, seed=31))
    full = fa.forward_flash2(q, k, v, 0.125, True)
    P = 4
    per = (B * H) // P
    parts = []
    for r in range(P):
        sl = slice(r * per, (r + 1) * per)
        qs, ks, vs = (t.view(B * H, 1, N, 64)[sl] for t in (q, k, v))
        parts.append(fa.forward_flash2(qs.contiguous(), ks.contiguous(), vs.contiguous(), 0.125, True))
    assert torch.equal(torch.cat(parts).view(B, H, N, 64), full)


@pytest.mark.slow
def test_config4_sampled_rows(cuda):
    """Config 4 shape on a subset of slices (B=16,H=32 would be 512 slices);
    the rows checked are sampled, which is exact since rows are independent."""
    S, N = 8, 8192
    q, k, v = orc.make_qkv(1, S, N, 64, seed=4)
    out = fa.forward_flash2(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, True).cpu()
    rows = torch.tensor([0, 1, 127, 128, 4095, 4096, 8000, 8191])
    ref = orc.attention_rows_fp32(q.view(S, N, 64), k.view(S, N, 64), v.view(S, N, 64), rows, 0.125, True)
    _check(out.view(S, N, 64)[:, rows], ref, "config4 rows")


def test_concurrent_python_threads(cuda):
    # the binding releases the GIL around the launch: calls from several
    # threads, each on its own stream, give the single-thread result
    import threading

    q, k, v = (t.to(cuda) for t in orc.make_qkv(2, 8, 1024, 64, seed=31))
    ref = fa.forward_flash2(q, k, v, 0.0, True)
    torch.cuda.synchronize()
    results, errors = [None] * 4, []

    def work(i):
        try:
            s = torch.cuda.Stream(cuda)
            with torch.cuda.stream(s):
                outs = [fa.forward_flash2(q, k, v, 0.0, True) for _ in range(50)]
            s.synchronize()
            results[i] = outs[-1]
        except Exception as e:  # surfaced in the main thread below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert fa.device_error() == 0
    for r in results:
        assert torch.equal(r, ref)
