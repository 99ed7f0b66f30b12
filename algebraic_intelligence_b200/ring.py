"""Ring (sequence-parallel) AFA across the GPUs of one node.

Reference: ``distributed_ring_afa`` (src/kernels/pallas_afa.py:618-662). Every
rank keeps its query shard; K/V shards travel one step around the ring per hop
(``lax.ppermute``, :651-652); each hop's unnormalised numerator and row sum are
added to the rank's accumulators (:648-649); one divide at the end (:661). AFA
needs no running-max rescale, so the merge is plain addition.

B200 form:
* one process per GPU; the K/V shard is packed as one (2, B, H, S, D) buffer
  and rotated with an NCCL send/recv pair (``torch.distributed`` P2P over
  NVLink/NVSwitch) issued *before* the hop's kernel, so the transfer of the
  next shard overlaps the compute on the current one (double buffer);
* a hop is one launch of the grouped forward kernel (``afa_fwd_hop``): the
  first hop stores the accumulators, middle hops add, and the last hop adds and
  divides in its epilogue -- no separate normalisation pass;
* ``layout="zigzag"`` (default for causal work) cuts the sequence into 2P
  chunks and gives rank r chunks r and 2P-1-r, which balances causal work;
  fully masked (query, key) chunk pairs are skipped on the host and partially
  masked tiles are masked in-kernel on global positions. ``layout="contiguous"``
  is the reference's own sharding (rank r holds block r).
* no collective other than the ring P2P; no TMA multicast anywhere.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import _lib

__all__ = ["distributed_ring_afa", "shard_sequence", "unshard_sequence", "ring_plan", "RingHop", "local_segments"]

Segment = Tuple[int, int, int]  # (row0 in the local shard, length, global position of row0)


def local_segments(rank: int, world: int, seq_len: int, layout: str) -> List[Segment]:
    """Row segments of the local shard and their global positions."""
    if layout == "contiguous":
        if seq_len % world:
            raise ValueError(f"sequence length {seq_len} must be divisible by the ring size {world}")
        s = seq_len // world
        return [(0, s, rank * s)]
    if layout == "zigzag":
        if seq_len % (2 * world):
            raise ValueError(f"zigzag sharding needs the sequence length {seq_len} divisible by 2*{world}")
        c = seq_len // (2 * world)
        return [(0, c, rank * c), (c, c, (2 * world - 1 - rank) * c)]
    raise ValueError(f"unknown layout {layout!r} (expected 'contiguous' or 'zigzag')")


def shard_sequence(x: torch.Tensor, rank: int, world: int, layout: str = "zigzag", dim: int = 2) -> torch.Tensor:
    """The rank's shard of a global (..., L, D) tensor along ``dim``."""
    segs = local_segments(rank, world, x.shape[dim], layout)
    return torch.cat([x.narrow(dim, pos, n) for _, n, pos in segs], dim=dim).contiguous()


def unshard_sequence(shards: Sequence[torch.Tensor], layout: str = "zigzag", dim: int = 2) -> torch.Tensor:
    """Inverse of ``shard_sequence`` given every rank's shard (in rank order)."""
    world = len(shards)
    seq_len = sum(s.shape[dim] for s in shards)
    pieces = []
    for r, sh in enumerate(shards):
        for row0, n, pos in local_segments(r, world, seq_len, layout):
            pieces.append((pos, sh.narrow(dim, row0, n)))
    pieces.sort(key=lambda t: t[0])
    return torch.cat([p for _, p in pieces], dim=dim)


@dataclass
class RingHop:
    src: int                      # rank whose K/V shard is processed in this hop
    mode: int                     # AFA_HOP_* for afa_fwd_hop
    problems: list                # [(q_row0, q_len, q_pos0, [(k_row0, k_len, k_pos0), ...]), ...]


def _visibility(q: Segment, k: Segment, causal: bool) -> str:
    """'full', 'partial' or 'none' for keys k seen from queries q."""
    if not causal:
        return "full"
    _, qn, qp = q
    _, kn, kp = k
    if kp > qp + qn - 1:
        return "none"
    if kp + kn - 1 <= qp:
        return "full"
    return "partial"


def ring_plan(rank: int, world: int, seq_len: int, causal: bool, layout: str) -> List[RingHop]:
    """The hops rank ``rank`` runs: which K/V shard, which (query, key) segment
    pairs, and the accumulator mode. Pure host logic."""
    qsegs = local_segments(rank, world, seq_len, layout)
    hops = []
    for hop in range(world):
        src = (rank - hop) % world
        ksegs = local_segments(src, world, seq_len, layout)
        if world == 1:
            mode = _lib.AFA_HOP_ONLY
        elif hop == 0:
            mode = _lib.AFA_HOP_STORE
        elif hop == world - 1:
            mode = _lib.AFA_HOP_FINALIZE
        else:
            mode = _lib.AFA_HOP_ACCUMULATE
        problems = []
        for qs in qsegs:
            vis = [(k, _visibility(qs, k, causal)) for k in ksegs]
            full = [k for k, v in vis if v == "full"]
            part = [k for k, v in vis if v == "partial"]
            if len(part) > 1:
                raise ValueError("ring layout produced two partially visible key segments for one query segment")
            keys = full + part
            if len(keys) > 2:
                raise ValueError("ring layout produced more than two key segments for one query segment")
            if not keys:
                if mode in (_lib.AFA_HOP_FINALIZE, _lib.AFA_HOP_ONLY):
                    # Nothing to add, but the rows still need their final divide:
                    # a wholly masked segment runs no tiles and only the epilogue.
                    keys = [ksegs[-1]]
                elif mode == _lib.AFA_HOP_STORE:
                    raise ValueError("every query segment must see keys in the first hop")
                else:
                    continue
            problems.append((qs[0], qs[1], qs[2], keys))
        hops.append(RingHop(src=src, mode=mode, problems=problems))
    return hops


def _p2p_rotate(send_buf: torch.Tensor, recv_buf: torch.Tensor, rank: int, world: int, group):
    """Start the ring step: send to rank+1, receive from rank-1 (ppermute)."""
    import torch.distributed as dist
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
    nxt = ranks[(rank + 1) % world]
    prv = ranks[(rank - 1) % world]
    ops = [dist.P2POp(dist.isend, send_buf, nxt, group), dist.P2POp(dist.irecv, recv_buf, prv, group)]
    return dist.batch_isend_irecv(ops)


def ring_loop(q: torch.Tensor, kv: torch.Tensor, hops: List[RingHop], compute: Callable,
              rotate: Optional[Callable]) -> None:
    """Drive the hops: start the next rotation, compute the current hop, wait.

    ``compute(hop, k, v)`` runs one hop on the current K/V; ``rotate(send,
    recv)`` starts the transfer and returns objects with ``wait()``.
    """
    bufs = [kv, torch.empty_like(kv) if len(hops) > 1 else None]
    for i, hop in enumerate(hops):
        cur = bufs[i % 2]
        reqs = rotate(cur, bufs[(i + 1) % 2]) if (i + 1 < len(hops)) else None
        if hop.problems:
            compute(hop, cur[0], cur[1])
        if reqs is not None:
            for r in reqs:
                r.wait()


def distributed_ring_afa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sink_omega: float = 0.5,
                         causal: bool = False, axis_name=None, num_devices: Optional[int] = None,
                         layout: str = "contiguous", return_denominator: bool = False):
    """Ring AFA over the ranks of a process group (src/kernels/pallas_afa.py:618-662).

    Call on every rank with that rank's shards q, k, v of shape
    (B, H, L/P, D) (``shard_sequence`` cuts them). ``axis_name`` is the
    ``torch.distributed`` process group of the ring (None = the default group),
    ``num_devices`` its size (checked when given). ``layout`` says how the
    global sequence was sharded: ``"contiguous"`` (the reference's layout) or
    ``"zigzag"`` (load-balanced causal). Returns the rank's output shard.
    """
    import torch.distributed as dist

    if q.ndim != 4 or tuple(q.shape) != tuple(k.shape) or tuple(q.shape) != tuple(v.shape):
        raise ValueError("q, k, and v must have the same four-dimensional shape")
    if not 0.0 <= float(sink_omega) < float("inf"):
        raise ValueError("sink_omega must be finite and nonnegative")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("ring AFA runs on CUDA tensors (one GPU per rank)")
    group = axis_name
    if dist.is_available() and dist.is_initialized():
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
    else:
        world, rank = 1, 0
    if num_devices is not None and num_devices != world:
        raise ValueError(f"num_devices={num_devices} but the ring has {world} ranks")
    b, h, s, d = q.shape
    seq_len = s * world
    hops = ring_plan(rank, world, seq_len, causal, layout)
    q = q.contiguous()
    kv = torch.stack([k, v]).contiguous()
    acc_dt = _lib.accum_dtype(q.dtype)
    out = torch.empty_like(q)
    den = torch.empty((b, h, s, 1), dtype=acc_dt, device=q.device)
    o_acc = torch.empty((b, h, s, d), dtype=acc_dt, device=q.device) if world > 1 else None
    d_acc = torch.empty((b, h, s), dtype=acc_dt, device=q.device) if world > 1 else None

    from .afa import hop_forward

    def compute(hop: RingHop, kk: torch.Tensor, vv: torch.Tensor) -> None:
        hop_forward(q, kk, vv, hop.problems, causal, hop.mode, o_acc=o_acc, d_acc=d_acc, out=out, d_total=den,
                    sink_omega=sink_omega)

    rotate = None
    if world > 1:
        rotate = lambda send, recv: _p2p_rotate(send, recv, rank, world, group)  # noqa: E731
    ring_loop(q, kv, hops, compute, rotate)
    if return_denominator:
        return out, den
    return out
