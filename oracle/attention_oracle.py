"""CPU oracle for the FlashLite FA2 forward path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this file;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and ``--impl reference`` legs use it, always as the checker or the CPU
baseline, never as the thing measured on the GPU.

What it restates (thebigblender/FlashLite, paths relative to that repo):

* ``attention_fp32``: the reference's attention mathematics in fp32 on host
  cores: softmax((Q K^T) * sm_scale [causal: keys j > i masked]) V with fp16
  inputs upcast to fp32. Follows ``benchmarks/benchmark_throughput.py:174-177``
  (``unfused_attn``) and the formulation in ``csrc/kernel_naive.cu:106-114``;
  ``sm_scale == 0`` means 1/sqrt(D) (``csrc/kernel_flash2.cu:769-771``).
* ``flash2_tiled_reference``: the reference kernel's own tiled algorithm and
  rounding (``csrc/kernel_flash2.cu:141-386``): log2(e) prescale (:772),
  -1e30 sentinel masking (:197-230), rescale = exp2(m_prev - m_new) or 0 when
  m_prev is the sentinel (:250-254), P rounded to fp16 before P·V while l
  sums the unrounded fp32 p (:278-294, :339), O * (1/l or 0) (:364-369).
  Used to show the tolerance is met by the reference's own numerics.
* ``flops``: ``benchmarks/benchmark_throughput.py:23-31``.
* ``attention_backward_fp32``: gradients of ``attention_fp32`` (no reference
  counterpart: the reference is forward-only). The standard softmax-attention
  backward (FlashAttention-2, Dao 2023, Algorithm 2): dV = P^T dO,
  dP = dO V^T, D_i = rowsum(dO_i * O_i), dS = P * (dP - D),
  dQ = scale dS K, dK = scale dS^T Q, in fp32. Pinned against
  ``torch.autograd`` in ``tests/test_oracle.py``.

Pinning: ``tests/test_oracle.py`` checks ``attention_fp32`` against
``torch.nn.functional.scaled_dot_product_attention`` (the reference tests'
oracle, ``tests/test_correctness.py:43-45,75-77``) on the reference test
matrix and against the committed golden vectors in ``tests/golden/``.
"""
from __future__ import annotations

import math

import numpy as np
import torch

LOG2_E = 1.44269504088896340736


def default_scale(head_dim: int, sm_scale: float) -> float:
    """csrc/kernel_flash2.cu:769-771: 0 selects 1/sqrt(D) (computed in fp32)."""
    if sm_scale == 0.0:
        return float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
    return float(sm_scale)


def flops(B: int, H: int, N: int, D: int, causal: bool) -> float:
    """benchmarks/benchmark_throughput.py:23-31: 4·B·H·N²·D, halved for causal."""
    return (2.0 if causal else 4.0) * B * H * N * N * D


def make_qkv(B: int, H: int, N: int, D: int, seed: int, scale: float = 1.0,
             slices: range | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Seeded i.i.d. N(0,1)·scale fp16 Q, K, V on the host, shape [B,H,N,D].

    Each (b,h) slice draws from its own generator (seed, slice index), so a
    contiguous range of slices (``slices``; returned as [len, 1, N, D]) can be
    generated on any rank without materialising the rest, and the values do
    not depend on how slices are sharded.
    """
    idx = range(B * H) if slices is None else slices
    out = []
    for name in range(3):
        t = torch.empty(len(idx), N, D, dtype=torch.float16)
        for r, s in enumerate(idx):
            g = torch.Generator().manual_seed((seed * 1_000_003 + s) * 4 + name)
            t[r] = (torch.randn(N, D, generator=g, dtype=torch.float32) * scale).to(torch.float16)
        out.append(t)
    if slices is None:
        return tuple(x.view(B, H, N, D) for x in out)  # type: ignore[return-value]
    return tuple(x.view(len(idx), 1, N, D) for x in out)  # type: ignore[return-value]


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float = 0.0,
                   is_causal: bool = False) -> torch.Tensor:
    """Exact fp32 attention on host cores; returns fp32 [B,H,N,D]."""
    D = q.shape[-1]
    scale = default_scale(D, sm_scale)
    qf, kf, vf = (t.detach().to("cpu", torch.float32) for t in (q, k, v))
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    if is_causal:
        n, m = s.shape[-2], s.shape[-1]
        mask = torch.ones(n, m, dtype=torch.bool).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, vf)


def attention_backward_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, do: torch.Tensor,
                            sm_scale: float = 0.0, is_causal: bool = False):
    """fp32 gradients (dq, dk, dv) of attention_fp32 for the output gradient do."""
    D = q.shape[-1]
    scale = default_scale(D, sm_scale)
    qf, kf, vf, dof = (t.detach().to("cpu", torch.float32) for t in (q, k, v, do))
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    if is_causal:
        n, m = s.shape[-2], s.shape[-1]
        s = s.masked_fill(torch.ones(n, m, dtype=torch.bool).triu(1), float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, vf)
    dv = torch.matmul(p.transpose(-2, -1), dof)
    dp = torch.matmul(dof, vf.transpose(-2, -1))
    delta = (dof * o).sum(dim=-1, keepdim=True)
    ds = p * (dp - delta)
    dq = torch.matmul(ds, kf) * scale
    dk = torch.matmul(ds.transpose(-2, -1), qf) * scale
    return dq, dk, dv


def grad_error_metrics(got: torch.Tensor, ref: torch.Tensor) -> tuple[float, float]:
    """(max-abs error / max |ref|, mean-abs error / mean |ref|) of a gradient."""
    g = got.detach().to("cpu", torch.float32)
    r = ref.detach().to("cpu", torch.float32)
    err = (g - r).abs()
    return (err.max().item() / max(r.abs().max().item(), 1e-30),
            err.mean().item() / max(r.abs().mean().item(), 1e-30))


def attention_rows_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows,
                        sm_scale: float = 0.0, is_causal: bool = False) -> torch.Tensor:
    """fp32 attention for selected query rows only (each row is independent).

    q, k, v: [S, N, D] (one tensor per (b,h) slice stacked); rows: 1-D index
    tensor of query positions. Returns fp32 [S, len(rows), D].
    """
    D = q.shape[-1]
    scale = default_scale(D, sm_scale)
    rows = torch.as_tensor(rows, dtype=torch.long)
    qf = q.detach().to("cpu", torch.float32)[..., rows, :]
    kf, vf = (t.detach().to("cpu", torch.float32) for t in (k, v))
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    if is_causal:
        keys = torch.arange(k.shape[-2])
        s = s.masked_fill(keys[None, :] > rows[:, None], float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), vf)


def block_attention_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_offset: int,
                        kv_offset: int, sm_scale: float, is_causal: bool):
    """Attention of a query block against one key/value block (ring step).

    Returns (o, lse): o fp32 normalised within the block, lse fp32 natural
    log-sum-exp of the scaled scores; rows without a visible key give
    (0, -inf). Shapes: q [..., Nq, D], k/v [..., Nk, D].
    """
    D = q.shape[-1]
    scale = default_scale(D, sm_scale)
    qf, kf, vf = (t.detach().to("cpu", torch.float32) for t in (q, k, v))
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    if is_causal:
        qpos = torch.arange(q.shape[-2]) + q_offset
        kpos = torch.arange(k.shape[-2]) + kv_offset
        s = s.masked_fill(kpos[None, :] > qpos[:, None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[..., None])
    o = torch.matmul(p, vf)
    return o, lse


def merge_lse(o_a: torch.Tensor, lse_a: torch.Tensor, o_b: torch.Tensor, lse_b: torch.Tensor):
    """Combine two normalised partial results by log-sum-exp weights."""
    mx = torch.maximum(lse_a, lse_b)
    safe = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
    wa = torch.exp(lse_a - safe)
    wb = torch.exp(lse_b - safe)
    tot = wa + wb
    lse = torch.where(tot > 0, safe + torch.log(tot), torch.full_like(tot, float("-inf")))
    denom = torch.where(tot > 0, tot, torch.ones_like(tot))
    o = (o_a * wa[..., None] + o_b * wb[..., None]) / denom[..., None]
    return o, lse


def flash2_tiled_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           sm_scale: float = 0.0, is_causal: bool = False) -> np.ndarray:
    """Restatement of the reference FA2 kernel's tiled algorithm (numpy, fp32).

    Br = 128 when N >= 2048 else 64 (csrc/kernel_flash2.cu:789-835), Bc = 64.
    Returns fp16 [B,H,N,D] as a numpy array. Vectorised over the rows of a
    query tile; meant for N up to a few thousand.
    """
    B, H, N, D = q.shape
    scale = default_scale(D, sm_scale)
    sl2 = np.float32(scale * LOG2_E)
    br, bc = (128 if N >= 2048 else 64), 64
    qn = q.detach().cpu().numpy().astype(np.float32)
    kn = k.detach().cpu().numpy().astype(np.float32)
    vn = v.detach().cpu().numpy().astype(np.float32)
    out = np.zeros((B, H, N, D), dtype=np.float16)
    sent = np.float32(-1e30)
    n_kv = (N + bc - 1) // bc
    for b in range(B):
        for h in range(H):
            for qs in range(0, N, br):
                rows = np.arange(qs, qs + br)
                qt = np.zeros((br, D), np.float32)
                valid_r = rows < N
                qt[valid_r] = qn[b, h, rows[valid_r]]
                m = np.full(br, sent, np.float32)
                l = np.zeros(br, np.float32)
                o = np.zeros((br, D), np.float32)
                tiles = min(n_kv, (qs + br - 1) // bc + 1) if is_causal else n_kv
                for j in range(tiles):
                    ks = j * bc
                    cols = np.arange(ks, ks + bc)
                    kt = np.zeros((bc, D), np.float32)
                    vt = np.zeros((bc, D), np.float32)
                    vc = cols < N
                    kt[vc] = kn[b, h, cols[vc]]
                    vt[vc] = vn[b, h, cols[vc]]
                    s = (qt @ kt.T).astype(np.float32)
                    ok = (cols[None, :] < N) & valid_r[:, None]
                    if is_causal:
                        ok &= cols[None, :] <= rows[:, None]
                    s = np.where(ok, s * sl2, sent).astype(np.float32)
                    m_new = np.maximum(m, s.max(axis=1))
                    resc = np.where(m > np.float32(-1e20), np.exp2(m - m_new), 0).astype(np.float32)
                    p = np.where(s > np.float32(-1e20), np.exp2(s - m_new[:, None]), 0).astype(np.float32)
                    l = l * resc + p.sum(axis=1, dtype=np.float32)
                    o = o * resc[:, None] + p.astype(np.float16).astype(np.float32) @ vt
                    m = m_new
                inv = np.where(l > 0, 1.0 / np.where(l > 0, l, 1), 0).astype(np.float32)
                res = (o * inv[:, None]).astype(np.float16)
                out[b, h, rows[valid_r]] = res[valid_r]
    return out


def error_metrics(out: torch.Tensor, ref: torch.Tensor) -> tuple[float, float]:
    """(max-abs, mean-abs) error of out against ref, both upcast to fp32."""
    d = (out.detach().to("cpu", torch.float32) - ref.detach().to("cpu", torch.float32)).abs()
    if d.numel() == 0:
        return 0.0, 0.0
    return float(d.max()), float(d.mean())


# Tolerances stated by the north star for this path (fp32 oracle vs kernel).
MAX_ABS_TOL = 2e-3
MEAN_ABS_TOL = 2e-4


def cpu_threads() -> int:
    return torch.get_num_threads()


def time_attention_fp32(q, k, v, sm_scale, is_causal, reps: int = 3) -> float:
    """Median wall time (s) of attention_fp32 over reps (CPU baseline)."""
    import time

    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        attention_fp32(q, k, v, sm_scale, is_causal)
        ts.append(time.perf_counter() - t0)
    ts.sort()
    return ts[len(ts) // 2]


__all__ = [
    "LOG2_E", "default_scale", "flops", "make_qkv", "attention_fp32", "attention_rows_fp32",
    "block_attention_lse", "merge_lse", "flash2_tiled_reference", "error_metrics",
    "MAX_ABS_TOL", "MEAN_ABS_TOL", "cpu_threads", "time_attention_fp32", "math",
]
