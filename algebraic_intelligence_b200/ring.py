"""Ring (sequence-parallel) AFA across the GPUs of one node.

Reference: ``distributed_ring_afa`` (src/kernels/pallas_afa.py:618-662). Every
rank keeps its query shard; K/V shards travel one step around the ring per hop
(``lax.ppermute``, :651-652); each hop's unnormalised numerator and row sum are
added to the rank's accumulators (:648-649); one divide at the end (:661). AFA
needs no running-max rescale, so the merge is plain addition.

B200 form:
* one process per GPU; each call publishes the rank's K/V shard as one
  (2, B, H, S, D) buffer that every rank maps with CUDA IPC, and hop i pulls
  the shard of rank ``hop.src`` straight from its owner with the copy engines
  (``CudaIpcExchange``): over NVSwitch every GPU reaches every other at full
  bandwidth, so the shard need not pass through the ranks in between. The
  pull for hop i+1 overlaps hop i's kernel and uses no SM; a call needs two
  stream-ordered barriers (after the publish, at the end) instead of a
  send/receive pair per hop;
* a hop is one launch of the grouped forward kernel (``afa_fwd_hop``): the
  first hop stores the accumulators, middle hops add, and the last hop adds and
  divides. On the tensor cores two consecutive middle hops share one launch
  (``launch_groups``): their shards are pulled side by side into one receive
  buffer, so the fixed cost of a launch (prologue, split tail, drain) is paid
  once for both;
* ``layout="zigzag"`` (default for causal work) cuts the sequence into 2P
  chunks and gives rank r chunks r and 2P-1-r, which balances causal work;
  fully masked (query, key) chunk pairs are skipped on the host and partially
  masked tiles are masked in-kernel on global positions. ``layout="contiguous"``
  is the reference's own sharding (rank r holds block r).
* no collective on the data path besides the two barriers; no TMA multicast anywhere.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import _lib

__all__ = ["distributed_ring_afa", "shard_sequence", "unshard_sequence", "ring_plan", "RingHop", "local_segments",
           "merge_hops", "launch_groups", "ring_loop", "KVExchange", "ListExchange", "CudaIpcExchange", "get_exchange",
           "release_ring_buffers"]

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


# Query pairs (256 rows) per (batch, head) that the persistent accumulate
# kernel plans (kMaxSkItems in csrc/afa_tc_shared.cuh); a larger launch runs
# the one-CTA-per-pair kernel, whose accumulate epilogue must not see one query
# row in two problems.
_SK_MAX_PAIRS = 1024
_MAX_PROBLEMS = 4


def merge_hops(group: Sequence[RingHop], shard_len: int) -> RingHop:
    """One launch for consecutive accumulate hops whose shards sit side by side
    in one receive buffer: hop j's keys at rows [j*shard_len, (j+1)*shard_len)
    of every (batch, head) block. Their partial sums only add, so the launch
    computes the same as the hops one after the other. A query segment's key
    segments from all the hops go into as few problems as the kernel takes
    (two key segments each, a partially visible one last), so its query pairs
    run long items; a segment with more keys than one problem holds appears in
    several problems, whose sums the persistent kernel adds."""
    keys_of = {}
    for j, h in enumerate(group):
        for qr, ql, qp, keys in h.problems:
            keys_of.setdefault((qr, ql, qp), []).extend((kr + j * shard_len, kl, kp) for kr, kl, kp in keys)
    problems = []
    for (qr, ql, qp), keys in keys_of.items():
        # Fully visible segments first: with causal masking only the second
        # segment of a problem may be partially visible.
        keys = sorted(keys, key=lambda k: k[2] + k[1] - 1 > qp)
        for i in range(0, len(keys), 2):
            problems.append((qr, ql, qp, keys[i:i + 2]))
    return RingHop(src=group[0].src, mode=group[0].mode, problems=problems)


def launch_groups(hops: Sequence[RingHop], shard_len: int, max_hops: int = 2):
    """The launches of one ring call: ``[(member hops, launched hop), ...]``.
    Wholly masked hops are left out (they pull and compute nothing). The
    first hop (STORE) and the last (FINALIZE) launch alone; consecutive
    accumulate hops are merged in pairs when ``max_hops`` allows it and the
    merged launch fits the persistent kernel (at most four problems and
    _SK_MAX_PAIRS query pairs per head), halving the per-launch prologue,
    split tail and drain of those hops."""
    live = [h for h in hops if h.problems]
    groups = []
    i = 0
    while i < len(live):
        h = live[i]
        if (max_hops > 1 and h.mode == _lib.AFA_HOP_ACCUMULATE and i + 1 < len(live)
                and live[i + 1].mode == _lib.AFA_HOP_ACCUMULATE):
            m = merge_hops(live[i:i + 2], shard_len)
            pairs = sum(-(-ql // 256) for _, ql, _, _ in m.problems)
            if len(m.problems) <= _MAX_PROBLEMS and pairs <= _SK_MAX_PAIRS:
                groups.append((list(live[i:i + 2]), m))
                i += 2
                continue
        groups.append(([h], h))
        i += 1
    return groups


class KVExchange:
    """How the hops of one ring call obtain their K/V shards.

    ``ring_loop`` drives it: ``publish`` makes this rank's shard readable by
    every rank of the ring and returns the local K and V that hop 0 reads
    (anything indexable as [0] = K, [1] = V);
    ``pull(src, slot)`` starts copying rank ``src``'s published shard into
    receive slot ``slot`` (0 or 1) and returns a token; ``ready(token)`` waits
    for that copy and returns the slot's tensor; ``finish`` ends the call.
    Transports with ``max_group`` > 1 also have ``pull_group(srcs, slot)``: the
    shards of ``srcs`` side by side along the sequence (rows
    [j*S, (j+1)*S) of every (batch, head) block hold srcs[j]'s), for one launch
    of merged hops (``launch_groups``). Subclasses are the transports.
    """

    rank = 0
    max_group = 1

    def publish(self, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def pull(self, src: int, slot: int):
        raise NotImplementedError

    def ready(self, token) -> torch.Tensor:
        raise NotImplementedError

    def finish(self) -> None:
        pass


class ListExchange(KVExchange):
    """Every rank's shard already lives in this process (a ring emulated in one
    process, rank by rank): ``shards[r]`` is rank r's (2, B, H, S, D) K/V."""

    max_group = 2

    def __init__(self, rank: int, shards: Sequence[torch.Tensor]):
        self.rank = rank
        self.shards = list(shards)
        self.recv = [torch.empty_like(self.shards[rank]) for _ in range(2)]
        self.recv_n = {}

    def publish(self, k, v):
        return self.shards[self.rank]

    def pull(self, src, slot):
        self.recv[slot].copy_(self.shards[src])
        return slot

    def pull_group(self, srcs, slot):
        n = len(srcs)
        mine = self.shards[self.rank]
        s = mine.shape[3]
        if n not in self.recv_n:
            shape = mine.shape[:3] + (n * s,) + mine.shape[4:]
            self.recv_n[n] = [torch.empty(shape, dtype=mine.dtype, device=mine.device) for _ in range(2)]
        buf = self.recv_n[n][slot]
        for j, src in enumerate(srcs):
            buf[:, :, :, j * s:(j + 1) * s].copy_(self.shards[src])
        return ("group", n, slot)

    def ready(self, token):
        if isinstance(token, tuple) and token[0] == "group":
            return self.recv_n[token[1]][token[2]]
        return self.recv[token]


class CudaIpcExchange(KVExchange):
    """The ring transport on one node: CUDA IPC mappings and copy-engine pulls.

    Each rank owns one published buffer that every other rank maps once
    (``afa_ring_export`` / ``afa_ring_open``), and two receive slots. A call
    copies K and V into the published buffer and runs a stream-ordered barrier
    (a one-element all-reduce on the group), after which every rank's shard is
    readable. Hop i then pulls the shard of rank ``hop.src`` with
    ``afa_ring_pull`` on a copy stream: the copy engines move it over NVLink
    while hop i-1's kernel runs, and no SM is taken from the kernel. The call
    ends with the compute stream joining the copy stream and a second barrier,
    so no rank's stream passes the end of a call (or the next call's publish)
    while any rank still reads its buffer -- a rank can free its memory or exit
    once its stream is synchronised.

    The publish copy and its barrier run on a side stream while hop 0's kernel
    reads the caller's K and V directly, so neither sits on the critical path.

    Ordering inside a rank: the publish waits for the compute stream (K and V
    written, the previous call's trailing barrier passed); a pull waits for the
    publish barrier and for the kernel that last read its slot (an event on the
    compute stream); a hop's kernel waits for its pull (an event on the copy
    stream); the trailing barrier follows the copy and side streams.

    One instance serves one (group, shape, dtype, device); ``get_exchange``
    caches them for the life of the process (``release_ring_buffers`` drops
    them). Buffers come from PyTorch's default caching allocator, which is built
    on cudaMalloc as CUDA IPC requires.
    """

    def __init__(self, shape, dtype: torch.dtype, device: torch.device, group=None, copy_streams: int = 1):
        import ctypes

        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        lib = _lib.load()
        kv_shape = (2,) + tuple(shape)
        self._pub = torch.empty(kv_shape, dtype=dtype, device=self.device)          # [K, V]
        self._recv = torch.empty((2,) + kv_shape, dtype=dtype, device=self.device)  # [slot][K, V]
        self.nbytes = self._pub.numel() * self._pub.element_size()
        handle = (ctypes.c_ubyte * 64)()
        offset = ctypes.c_ulonglong(0)
        _lib.check(lib.afa_ring_export(self._pub.data_ptr(), handle, ctypes.byref(offset)), "afa_ring_export")
        mine = torch.tensor(list(bytes(handle)) + list(offset.value.to_bytes(8, "little")), dtype=torch.uint8,
                            device=self.device)
        every = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(every, mine, group=group)
        self._bases = []
        self._peer = []
        for j, t in enumerate(every):
            if j == self.rank:
                self._peer.append(self._pub.data_ptr())
                continue
            raw = bytes(t.cpu().tolist())
            base = ctypes.c_void_p()
            _lib.check(lib.afa_ring_open(raw[:64], ctypes.byref(base)), "afa_ring_open")
            self._bases.append(base.value)
            self._peer.append(base.value + int.from_bytes(raw[64:72], "little"))
        self._shape = tuple(shape)
        self._recv_n = {}  # receive slots for merged hops, by hop count: [slot] -> (2, B, H, n*S, D)
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._copy = [torch.cuda.Stream(self.device) for _ in range(max(1, copy_streams))]
        # The publish copy and its barrier run here, beside hop 0's kernel
        # (which reads the caller's own K and V); high priority, so their
        # kernels take the first SM slot that frees.
        self._side = torch.cuda.Stream(self.device, priority=-1)
        self._published = None

    def _barrier(self):
        import torch.distributed as dist
        dist.all_reduce(self._flag, group=self.group)   # stream-ordered on the current stream

    def publish(self, k, v):
        cur = torch.cuda.current_stream(self.device)
        self._side.wait_stream(cur)                     # k, v written; the last call's trailing barrier passed
        with torch.cuda.stream(self._side):
            self._pub[0].copy_(k)
            self._pub[1].copy_(v)
            self._barrier()                             # every rank has published
        self._published = torch.cuda.Event()
        self._published.record(self._side)
        k.record_stream(self._side)
        v.record_stream(self._side)
        return (k, v)                                   # hop 0 reads the caller's tensors meanwhile

    def pull(self, src, slot):
        lib = _lib.load()
        cur = torch.cuda.current_stream(self.device)
        released = torch.cuda.Event()
        released.record(cur)
        n = len(self._copy)
        step = -(-self.nbytes // (n * 256)) * 256
        dst0 = self._recv[slot].data_ptr()
        src0 = self._peer[src]
        done = []
        for i, s in enumerate(self._copy):
            lo = i * step
            size = min(step, self.nbytes - lo)
            if size <= 0:
                break
            s.wait_event(released)
            s.wait_event(self._published)
            _lib.check(lib.afa_ring_pull(dst0 + lo, src0 + lo, size, s.cuda_stream), "afa_ring_pull")
            ev = torch.cuda.Event()
            ev.record(s)
            done.append(ev)
        return slot, done

    max_group = 2

    def pull_group(self, srcs, slot):
        """The shards of ``srcs`` side by side in one receive slot: each K and V
        goes into its rows of every (batch, head) block with one strided copy
        (``afa_ring_pull2d``) on the copy stream."""
        lib = _lib.load()
        n = len(srcs)
        if n not in self._recv_n:
            b, h, s, d = self._shape
            self._recv_n[n] = torch.empty((2, 2, b, h, n * s, d), dtype=self._pub.dtype, device=self.device)
        buf = self._recv_n[n][slot]
        cur = torch.cuda.current_stream(self.device)
        released = torch.cuda.Event()
        released.record(cur)
        cs = self._copy[0]
        cs.wait_event(released)
        cs.wait_event(self._published)
        b, h, s, d = self._shape
        row = s * d * self._pub.element_size()   # one (batch, head) block of one shard's K (or V)
        for j, src in enumerate(srcs):
            for kv in (0, 1):
                dst = buf[kv].data_ptr() + j * row
                src_ptr = self._peer[src] + kv * (self.nbytes // 2)
                _lib.check(lib.afa_ring_pull2d(dst, n * row, src_ptr, row, row, b * h, cs.cuda_stream),
                           "afa_ring_pull2d")
        ev = torch.cuda.Event()
        ev.record(cs)
        return ("group", n, slot, [ev])

    def ready(self, token):
        if token[0] == "group":
            _, n, slot, done = token
            buf = self._recv_n[n][slot]
        else:
            slot, done = token
            buf = self._recv[slot]
        cur = torch.cuda.current_stream(self.device)
        for ev in done:
            cur.wait_event(ev)
        return buf

    def finish(self):
        cur = torch.cuda.current_stream(self.device)
        for s in self._copy:
            cur.wait_stream(s)
        cur.wait_stream(self._side)
        self._barrier()                                 # every rank is done reading every buffer

    def close(self) -> None:
        """Unmaps the peers' buffers (after the device finished this rank's work;
        the trailing barrier of the last call already waited for every peer)."""
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        for b in self._bases:
            lib.afa_ring_close(b)
        self._bases = []
        self._peer = []


_EXCHANGES = {}


def get_exchange(shape, dtype: torch.dtype, device: torch.device, group=None) -> CudaIpcExchange:
    """The cached exchange of ``group`` for K/V shards of ``shape`` (B, H, S, D).
    The first call for a key is collective over the group (it swaps IPC handles).

    The key holds the process-group object itself (the default group's current
    object when ``group`` is None), so a group that is destroyed and created
    again never finds the old group's mappings.
    """
    import torch.distributed as dist
    device = torch.device(device)
    pg = group if group is not None else dist.group.WORLD
    key = (pg, tuple(shape), dtype, device.index)
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = CudaIpcExchange(shape, dtype, device, group)
    return ex


def release_ring_buffers() -> None:
    """Unmaps the peers' buffers and drops every cached exchange (and with them
    the published buffers). Call it on every rank once no rank runs ring calls
    any more."""
    for ex in _EXCHANGES.values():
        ex.close()
    _EXCHANGES.clear()


def ring_loop(k: torch.Tensor, v: torch.Tensor, hops: List[RingHop], compute: Callable,
              exchange: Optional[KVExchange], merge: Optional[bool] = None) -> None:
    """Drive the hops of one ring call.

    ``compute(hop, k, v)`` runs one launch (``launch_groups``: one hop, or two
    merged accumulate hops when the exchange can pull two shards into one
    buffer) on that launch's K/V. The first launch reads this rank's own shard;
    later ones pull the shards of their hops' ``src`` ranks from their owners,
    the pull for launch g+1 starting before launch g's compute so the two
    overlap (two receive slots). Wholly masked hops pull and compute nothing.
    With one rank (``exchange`` None) the only hop reads k and v. ``merge``
    None merges where the launches run on the tensor cores (bf16, head_dim 64
    or 128); True or False forces it (tests of the protocol use small shapes).
    """
    if exchange is None:
        for hop in hops:
            if hop.problems:
                compute(hop, k, v)
        return
    local = exchange.publish(k, v)
    if hops and hops[0].src != exchange.rank:
        raise ValueError("the first hop of a ring plan must read the rank's own shard")
    # Only the tensor cores' persistent accumulate kernel adds one query row's
    # partial sums from two problems of a launch (fire-and-forget reductions);
    # the CUDA-core kernels read-modify-write them, so their hops stay apart.
    if merge is None:
        merge = k.dtype == torch.bfloat16 and k.shape[3] in (64, 128)
    groups = launch_groups(hops, k.shape[2], getattr(exchange, "max_group", 1) if merge else 1)

    def start(g):
        if 0 < g < len(groups):
            members = groups[g][0]
            if len(members) == 1:
                return exchange.pull(members[0].src, g % 2)
            return exchange.pull_group([h.src for h in members], g % 2)
        return None

    pending = None
    for g, (_members, hop) in enumerate(groups):
        kv = local if g == 0 else exchange.ready(pending)
        pending = start(g + 1)
        compute(hop, kv[0], kv[1])
    exchange.finish()


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
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k and v must share a dtype, got {q.dtype}, {k.dtype} and {v.dtype}")
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
    acc_dt = _lib.accum_dtype(q.dtype)
    out = torch.empty_like(q)
    den = torch.empty((b, h, s, 1), dtype=acc_dt, device=q.device)
    o_acc = torch.empty((b, h, s, d), dtype=acc_dt, device=q.device) if world > 1 else None
    d_acc = torch.empty((b, h, s), dtype=acc_dt, device=q.device) if world > 1 else None

    from .afa import hop_forward

    def compute(hop: RingHop, kk: torch.Tensor, vv: torch.Tensor) -> None:
        hop_forward(q, kk, vv, hop.problems, causal, hop.mode, o_acc=o_acc, d_acc=d_acc, out=out, d_total=den,
                    sink_omega=sink_omega)

    exchange = get_exchange(q.shape, q.dtype, q.device, group) if world > 1 else None
    ring_loop(k.contiguous(), v.contiguous(), hops, compute, exchange)
    if return_denominator:
        return out, den
    return out
