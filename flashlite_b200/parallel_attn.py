"""Multi-GPU attention within one node: head sharding and ring attention.

Neither mode has a counterpart in the reference (thebigblender/FlashLite is
single-GPU; its only parallel axis is the CUDA grid, csrc/kernel_flash2.cu:791-792).
One process per GPU, ``torch.distributed`` for the plumbing.

* Head sharding: the B·H (b,h) slices of [B,H,N,D] are independent, so rank r
  takes a contiguous range of slices (``shard_range``) and runs the
  single-GPU kernel on it. No collective on the data path.
* Ring attention (sequence sharding): rank r holds query/key/value rows
  [r·Nb, (r+1)·Nb) of every head. K/V blocks travel P-1 hops around the ring
  (NCCL send/recv, double-buffered, issued before the block's compute so the
  transfer overlaps it). Each block step runs the FA2 kernel in "merge" mode,
  which folds the block's result into a running fp32 (O, log-sum-exp) state
  in its epilogue; with a causal mask, blocks from later ranks are skipped.
  A final cast writes fp16.
* Zig-zag ring (causal): the sequence is cut into 2P chunks and rank r holds
  chunks r and 2P-1-r, so every rank has the same causal work at every ring
  step (contiguous blocks cap the causal speed-up at P²/(2P-1); zig-zag
  removes the cap). Each step computes the visible (query chunk, key chunk)
  pairs of the two local query chunks against the two received key chunks.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> range:
    """Contiguous split of ``total`` items over ``world`` ranks; the first
    ``total % world`` ranks take one extra item."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("invalid world/rank")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def head_sharded_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float = 0.0,
                         is_causal: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Forward of this rank's contiguous (b,h) slice range; no communication.

    q, k, v are the local slices ([S, 1, N, D] or any [B', H', N, D]).
    """
    from . import flash_attn_wmma as fa

    return fa.forward_flash2(q, k, v, sm_scale, is_causal, out=out)


BlockFn = Callable[..., None]


def _step_events(events: Optional[list]):
    """Three timing events for one ring step (the first recorded now), or None."""
    if events is None:
        return None
    ev = tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
    ev[0].record()
    events.append(ev)
    return ev


def _record(ev, i: int) -> None:
    if ev is not None:
        ev[i].record()


def _default_block_fn():
    from . import flash_attn_wmma as fa

    return fa.forward_block, fa.ring_finalize


def ring_schedule(rank: int, world: int, causal: bool):
    """Per step s: (source block index, compute?) for this rank.

    At step s the rank holds the K/V block of rank (rank - s) mod world. With
    a causal mask over contiguous blocks, blocks from later ranks are fully
    masked and skipped (they are still forwarded around the ring).
    """
    steps = []
    for s in range(world):
        src = (rank - s) % world
        steps.append((src, (not causal) or src <= rank))
    return steps


class RingAttention:
    """Sequence-sharded attention forward over a process group.

    ``block_fn(q, k, v, o_acc, lse, q_offset, kv_offset, sm_scale, is_causal,
    first)`` merges one block into (o_acc, lse) in place and
    ``finalize_fn(o_acc, out)`` casts the result; both default to the CUDA
    kernels of this package (tests on CPU pass host implementations).
    """

    def __init__(self, group=None, block_fn: Optional[BlockFn] = None,
                 finalize_fn: Optional[Callable] = None):
        self.group = group
        if block_fn is None or finalize_fn is None:
            b, f = _default_block_fn()
            block_fn = block_fn or b
            finalize_fn = finalize_fn or f
        self.block_fn = block_fn
        self.finalize_fn = finalize_fn
        self._bufs = None

    def _buffers(self, k: torch.Tensor):
        key = (tuple(k.shape), k.dtype, k.device)
        if self._bufs is None or self._bufs[0] != key:
            self._bufs = (key, [torch.empty_like(k) for _ in range(4)])
        return self._bufs[1]

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float = 0.0,
                is_causal: bool = True, out: Optional[torch.Tensor] = None,
                o_acc: Optional[torch.Tensor] = None,
                lse: Optional[torch.Tensor] = None, events: Optional[list] = None) -> torch.Tensor:
        """``events``: if a list, one (start, computed, received) triple of
        timing CUDA events is appended per ring step, recorded on the current
        stream before the step's block compute, after it, and after the wait
        for the next K/V block (so received - computed is exchange time the
        compute did not hide)."""
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        if q.shape != k.shape or k.shape != v.shape:
            raise ValueError("ring attention expects q, k, v blocks of equal shape [B, H, Nb, D]")
        B, H, Nb, D = q.shape
        if o_acc is None:
            o_acc = torch.empty(B, H, Nb, D, dtype=torch.float32, device=q.device)
        if lse is None:
            lse = torch.empty(B, H, Nb, dtype=torch.float32, device=q.device)
        if out is None:
            out = torch.empty_like(q)
        nxt, prv = (rank + 1) % world, (rank - 1) % world
        g_nxt = dist.get_global_rank(self.group, nxt) if self.group is not None else nxt
        g_prv = dist.get_global_rank(self.group, prv) if self.group is not None else prv
        bufs = self._buffers(k)
        cur_k, cur_v = k, v
        for s, (src, compute) in enumerate(ring_schedule(rank, world, is_causal)):
            reqs = []
            if s < world - 1:
                nk, nv = bufs[2 * (s % 2)], bufs[2 * (s % 2) + 1]
                ops = [dist.P2POp(dist.isend, cur_k, g_nxt, self.group),
                       dist.P2POp(dist.isend, cur_v, g_nxt, self.group),
                       dist.P2POp(dist.irecv, nk, g_prv, self.group),
                       dist.P2POp(dist.irecv, nv, g_prv, self.group)]
                reqs = dist.batch_isend_irecv(ops)
            ev = _step_events(events)
            if compute:
                self.block_fn(q, cur_k, cur_v, o_acc, lse, rank * Nb, src * Nb, sm_scale,
                              is_causal, s == 0)
            _record(ev, 1)
            for r in reqs:
                r.wait()
            _record(ev, 2)
            if s < world - 1:
                cur_k, cur_v = nk, nv
        self.finalize_fn(o_acc, out)
        return out



def zigzag_chunks(rank: int, world: int) -> tuple:
    """Chunk indices (of 2·world equal chunks) held by ``rank``."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("invalid world/rank")
    return rank, 2 * world - 1 - rank


def zigzag_pairs(rank: int, src: int, world: int, causal: bool):
    """(query chunk slot, key chunk slot) pairs to compute when ``rank`` holds
    the key/value chunks of rank ``src``; slot 0 / 1 = the lower / upper chunk
    of a rank. Pairs whose keys all lie after the queries are left out."""
    qc, kc = zigzag_chunks(rank, world), zigzag_chunks(src, world)
    return [(a, b) for a in range(2) for b in range(2) if not causal or kc[b] <= qc[a]]


class ZigzagRingAttention(RingAttention):
    """Ring attention over the zig-zag layout (see module docstring).

    ``forward(q, k, v)`` takes this rank's two chunks as ``[2, B, H, c, D]``
    tensors (slot 0 = chunk r, slot 1 = chunk 2P-1-r) and returns the output
    in the same layout. The K/V of a rank travel as one contiguous
    ``[2 (k, v), 2 (slots), B, H, c, D]`` buffer.
    """

    def _kv_buffers(self, kv: torch.Tensor):
        key = (tuple(kv.shape), kv.dtype, kv.device, "zz")
        if self._bufs is None or self._bufs[0] != key:
            self._bufs = (key, [torch.empty_like(kv) for _ in range(2)])
        return self._bufs[1]

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float = 0.0,
                is_causal: bool = True, out: Optional[torch.Tensor] = None,
                o_acc: Optional[torch.Tensor] = None,
                lse: Optional[torch.Tensor] = None, events: Optional[list] = None) -> torch.Tensor:
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        if q.shape != k.shape or k.shape != v.shape or q.dim() != 5 or q.shape[0] != 2:
            raise ValueError("zig-zag ring attention expects q, k, v of shape [2, B, H, c, D]")
        _, B, H, c, D = q.shape
        if o_acc is None:
            o_acc = torch.empty(2, B, H, c, D, dtype=torch.float32, device=q.device)
        if lse is None:
            lse = torch.empty(2, B, H, c, dtype=torch.float32, device=q.device)
        if out is None:
            out = torch.empty_like(q)
        nxt, prv = (rank + 1) % world, (rank - 1) % world
        g_nxt = dist.get_global_rank(self.group, nxt) if self.group is not None else nxt
        g_prv = dist.get_global_rank(self.group, prv) if self.group is not None else prv
        bufs = self._kv_buffers(torch.stack((k, v)))
        cur = bufs[1]
        cur.copy_(torch.stack((k, v)))
        own = zigzag_chunks(rank, world)
        started = [False, False]
        for s in range(world):
            src = (rank - s) % world
            reqs = []
            if s < world - 1:
                nxt_buf = bufs[s % 2] if bufs[s % 2] is not cur else bufs[(s + 1) % 2]
                ops = [dist.P2POp(dist.isend, cur, g_nxt, self.group),
                       dist.P2POp(dist.irecv, nxt_buf, g_prv, self.group)]
                reqs = dist.batch_isend_irecv(ops)
            kc = zigzag_chunks(src, world)
            ev = _step_events(events)
            for a, b in zigzag_pairs(rank, src, world, is_causal):
                self.block_fn(q[a], cur[0, b], cur[1, b], o_acc[a], lse[a], own[a] * c, kc[b] * c,
                              sm_scale, is_causal, not started[a])
                started[a] = True
            _record(ev, 1)
            for r in reqs:
                r.wait()
            _record(ev, 2)
            if s < world - 1:
                cur = nxt_buf
        for a in range(2):
            self.finalize_fn(o_acc[a], out[a])
        return out
