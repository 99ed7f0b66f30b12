"""Host-side logic without a GPU: argument checks with the reference's exception
types and messages, and the ring plan (zigzag / contiguous sharding, hop modes,
the ring's K/V exchange protocol over gloo)."""
import os

import numpy as np
import pytest
import torch

import algebraic_intelligence_b200 as afa
from algebraic_intelligence_b200 import _lib
from algebraic_intelligence_b200.ring import (KVExchange, ListExchange, launch_groups, local_segments, ring_loop, ring_plan,
                                              shard_sequence, unshard_sequence)
from oracle import afa_oracle as orc


# ---------------------------------------------------------------------------
# Argument checks (src/kernels/pallas_afa.py:167-186, :342-353, :705-708;
# src/attention.py:60-63; src/primitives.py:17-21, 56-61)
# ---------------------------------------------------------------------------
def _x(shape, dtype=np.float32):
    return np.ones(shape, dtype=dtype)


@pytest.mark.parametrize("kwargs,match", [
    ({"q": _x((2, 64, 8))}, "must all have shape"),
    ({"k": _x((1, 1, 64, 16))}, "shapes must match"),
    ({"sink_omega": -1.0}, "sink_omega"),
    ({"sink_omega": float("nan")}, "sink_omega"),
    ({"block_q": 0}, "positive"),
    ({"q": _x((1, 1, 64, 192)), "k": _x((1, 1, 64, 192)), "v": _x((1, 1, 64, 192))}, "divisible by 128"),
    ({"block_q": 48}, "divisible by block_q"),
    ({"valid_seq_len": 0}, "valid_seq_len"),
    ({"valid_seq_len": 65}, "valid_seq_len"),
])
def test_pallas_afa_forward_value_errors(kwargs, match):
    args = {"q": _x((1, 1, 64, 8)), "k": _x((1, 1, 64, 8)), "v": _x((1, 1, 64, 8)), "block_q": 64, "block_k": 64}
    args.update(kwargs)
    with pytest.raises(ValueError, match=match):
        afa.pallas_afa_forward(**args)


def test_tiled_rejects_partial_tiles():
    # tests/test_pallas_afa.py:201-204
    x = _x((1, 1, 190, 32))
    with pytest.raises(ValueError, match="divisible"):
        afa.tiled_afa_forward(x, x, x, block_q=64, block_k=128)


def test_integer_inputs_are_type_errors():
    x = np.ones((1, 1, 64, 8), dtype=np.int32)
    with pytest.raises(TypeError):
        afa.pallas_afa_forward(x, x, x, block_q=64, block_k=64)
    with pytest.raises(TypeError):
        afa.algebraic_softmax(np.arange(4))


@pytest.mark.parametrize("kwargs", [{"sink_omega": -1.0}, {"sink_omega": float("nan")}, {"eps": 0.0},
                                    {"eps": -1.0}])
def test_softmax_invalid_hyperparameters(kwargs):
    # tests/test_attention.py:66-68
    with pytest.raises(ValueError):
        afa.algebraic_softmax(np.ones(4), **kwargs)


def test_softmax_invalid_input():
    # tests/test_attention.py:71-74
    with pytest.raises(TypeError):
        afa.algebraic_softmax(np.arange(4))
    with pytest.raises(ValueError):
        afa.algebraic_softmax(np.ones(()))
    with pytest.raises(ValueError):
        afa.algebraic_softmax(np.ones((2, 0)))


def test_unified_entry_value_errors():
    with pytest.raises(ValueError, match="same four-dimensional shape"):
        afa.algebraic_flash_attention(_x((1, 1, 64, 8)), _x((1, 1, 63, 8)), _x((1, 1, 64, 8)))
    with pytest.raises(ValueError, match="positive"):
        afa.algebraic_flash_attention(_x((1, 1, 64, 8)), _x((1, 1, 64, 8)), _x((1, 1, 64, 8)), block_k=-1)


def test_backward_argument_errors():
    x = _x((1, 1, 64, 8))
    d = np.ones((1, 1, 64, 1), dtype=np.float32)
    with pytest.raises(ValueError, match="same four-dimensional shape"):
        afa.tiled_afa_backward(x, x, x, _x((1, 1, 63, 8)), d, x)
    with pytest.raises(ValueError, match="positive"):
        afa.tiled_afa_backward(x, x, x, x, d, x, block_q=0)
    with pytest.raises(ValueError, match="d_total"):
        afa.tiled_afa_backward(x, x, x, x, np.ones((1, 1, 32, 1), dtype=np.float32), x)
    with pytest.raises(ValueError, match="valid_seq_len"):
        afa.tiled_afa_backward(x, x, x, x, d, x, valid_seq_len=65)
    xi = np.ones((1, 1, 64, 8), dtype=np.int32)
    with pytest.raises(TypeError):
        afa.tiled_afa_backward(xi, xi, xi, xi, d, xi)


def test_ago_argument_errors():
    """src/attention.py:175-178, :222-226."""
    with pytest.raises(ValueError, match="positive even"):
        afa.build_cayley_rotary_matrix(7, 16)
    with pytest.raises(ValueError, match="max_seq_len"):
        afa.build_cayley_rotary_matrix(8, 0)
    with pytest.raises(ValueError, match="freqs must have shape"):
        afa.build_cayley_rotary_matrix(8, 4, freqs=[0.5, 0.5])
    with pytest.raises(ValueError, match="shapes must match"):
        afa.apply_ago_rotations(np.ones((4, 8)), np.ones((4, 6)))
    with pytest.raises(ValueError, match="must be even"):
        afa.apply_ago_rotations(np.ones((4, 7)), np.ones((4, 7)))
    with pytest.raises(TypeError):
        afa.apply_ago_rotations(np.ones((4, 8), dtype=np.int32), np.ones((4, 8), dtype=np.int32))
    with pytest.raises(TypeError, match="Unsupported rotary"):
        from algebraic_intelligence_b200.ago import _extract_cs
        _extract_cs(3.0)


# ---------------------------------------------------------------------------
# Ring plan
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_shard_roundtrip(world, layout):
    x = torch.arange(2 * 3 * 16 * world * 2, dtype=torch.float32).reshape(2, 3, 16 * world, 2)
    shards = [shard_sequence(x, r, world, layout) for r in range(world)]
    assert torch.equal(unshard_sequence(shards, layout), x)


def _simulate_ring(q, k, v, world, causal, layout, sink=0.5):
    """Runs ring_plan + ring_loop for every rank in-process; the hop compute is
    the oracle (the checker), the exchange a list of every rank's shard."""
    seq = q.shape[2]
    qs = [shard_sequence(q, r, world, layout) for r in range(world)]
    kvs = [torch.stack([shard_sequence(k, r, world, layout), shard_sequence(v, r, world, layout)])
           for r in range(world)]
    outs = []
    for r in range(world):
        hops = ring_plan(r, world, seq, causal, layout)
        s = qs[r].shape[2]
        o_acc = np.zeros(qs[r].shape)
        d_acc = np.zeros(qs[r].shape[:3])
        out = np.full(qs[r].shape, np.nan)

        def compute(hop, kk, vv):
            assert torch.equal(torch.stack([kk, vv]), kvs[hop.src])
            for qr, ql, qp, segs in hop.problems:
                num = np.zeros(qs[r].shape[:2] + (ql, q.shape[3]))
                rs = np.zeros(qs[r].shape[:2] + (ql, 1))
                for kr, kl, kp in segs:
                    n_, r_ = orc.afa_blocked(qs[r][:, :, qr:qr + ql].numpy(), kk[:, :, kr:kr + kl].numpy(),
                                             vv[:, :, kr:kr + kl].numpy(), causal=causal, q_pos0=qp, k_pos0=kp,
                                             raw=True)
                    num += n_
                    rs += r_
                sl = slice(qr, qr + ql)
                if hop.mode == _lib.AFA_HOP_STORE:
                    o_acc[:, :, sl], d_acc[:, :, sl] = num, rs[..., 0]
                elif hop.mode == _lib.AFA_HOP_ACCUMULATE:
                    o_acc[:, :, sl] += num
                    d_acc[:, :, sl] += rs[..., 0]
                elif hop.mode == _lib.AFA_HOP_FINALIZE:
                    out[:, :, sl] = (o_acc[:, :, sl] + num) / (d_acc[:, :, sl] + rs[..., 0] + sink)[..., None]
                else:
                    out[:, :, sl] = num / (rs + sink)

        ex = ListExchange(r, kvs) if world > 1 else None
        ring_loop(kvs[r][0], kvs[r][1], hops, compute, ex)
        assert s == qs[r].shape[2]
        outs.append(torch.from_numpy(out))
    return unshard_sequence(outs, layout).numpy()


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_ring_plan_reproduces_global_afa(world, causal, layout):
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, 2, 16 * world, 8, generator=g, dtype=torch.float64) for _ in range(3))
    ring = _simulate_ring(q, k, v, world, causal, layout)
    assert np.all(np.isfinite(ring)), "a row was never finalised"
    assert orc.rel_err(ring, orc.afa(q.numpy(), k.numpy(), v.numpy(), causal=causal)) <= 1e-12


def test_zigzag_skips_masked_pairs_and_balances_work():
    world, seq = 8, 8 * 2 * 1024
    work = []
    for r in range(world):
        tiles = 0
        for hop in ring_plan(r, world, seq, True, "zigzag"):
            for qr, ql, qp, segs in hop.problems:
                for kr, kl, kp in segs:
                    # visible (query, key) pairs of this problem
                    qpos = np.arange(qp, qp + ql)
                    tiles += int(np.clip(qpos[:, None] - kp + 1, 0, kl).sum())
        work.append(tiles)
    assert max(work) == min(work), work
    assert sum(work) == seq * (seq + 1) // 2


def test_first_hop_covers_every_query_segment():
    for world in (2, 4, 8):
        for r in range(world):
            for layout in ("contiguous", "zigzag"):
                for causal in (False, True):
                    hops = ring_plan(r, world, 64 * world, causal, layout)
                    covered = {p[0] for p in hops[0].problems}
                    assert covered == {s[0] for s in local_segments(r, world, 64 * world, layout)}
                    last = {p[0] for p in hops[-1].problems}
                    assert last == covered  # every row gets its final divide


class _SharedMemoryExchange(KVExchange):
    """The CUDA IPC exchange's protocol on CPU processes: published buffers are
    shared-memory tensors every process maps, the barriers gloo barriers, a
    pull a copy out of the owner's buffer. ``pubs[r]`` is rank r's."""

    def __init__(self, rank, pubs, log, max_group=1):
        import torch.distributed as dist
        self.dist = dist
        self.rank = rank
        self.pubs = pubs
        self.recv = [torch.empty_like(pubs[rank]) for _ in range(2)]
        self.log = log
        self.max_group = max_group
        self.recv_n = {}

    def publish(self, k, v):
        buf = self.pubs[self.rank]
        buf[0].copy_(k)
        buf[1].copy_(v)
        self.dist.barrier()
        return buf

    def pull(self, src, slot):
        self.log.append(("pull", src, slot))
        self.recv[slot].copy_(self.pubs[src])
        return slot

    def pull_group(self, srcs, slot):
        self.log.append(("pull", tuple(srcs), slot))
        mine = self.pubs[self.rank]
        s = mine.shape[3]
        n = len(srcs)
        if n not in self.recv_n:
            self.recv_n[n] = [torch.empty(mine.shape[:3] + (n * s,) + mine.shape[4:]) for _ in range(2)]
        for j, src in enumerate(srcs):
            self.recv_n[n][slot][:, :, :, j * s:(j + 1) * s].copy_(self.pubs[src])
        return ("group", n, slot)

    def ready(self, token):
        if isinstance(token, tuple):
            return self.recv_n[token[1]][token[2]]
        return self.recv[token]

    def finish(self):
        self.log.append(("end",))
        self.dist.barrier()


def _gloo_worker(rank, world, port, pubs, causal, results, layout="contiguous", dtype=torch.float32, max_group=1):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        log = []
        ex = _SharedMemoryExchange(rank, pubs, log, max_group)
        hops = ring_plan(rank, world, 4 * world, causal, layout)
        seen = []
        for call in range(3):
            # K carries (call, rank) so a hop that read a stale or foreign buffer shows it.
            k = torch.full((1, 1, 4, 2), float(100 * call + rank), dtype=dtype)
            v = -k

            def compute(hop, kk, vv):
                # A merged launch sees its hops' shards side by side (4 rows each).
                assert torch.equal(vv, -kk)
                for j in range(kk.shape[2] // 4):
                    seen.append((call, int(kk[0, 0, 4 * j, 0]) - 100 * call, int(kk[0, 0, 4 * j, 0])))

            # No barrier between calls besides the exchange's own: they alone
            # must keep a fast rank from overwriting what a slow rank still reads.
            ring_loop(k, v, hops, compute, ex, merge=max_group > 1)
        results[rank] = (seen, log)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("causal", [False, True])
def test_ring_exchange_protocol_over_gloo(world, causal):
    """Real processes run the ring's publish / barrier / pull protocol over
    shared memory: every hop reads the shard of rank r-h of the same call (the
    ppermute order of pallas_afa.py:632, :651-652), wholly masked hops pull
    nothing, and every call ends with its barrier."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    pubs = [torch.zeros(2, 1, 1, 4, 2).share_memory_() for _ in range(world)]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, pubs, causal, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        seen, log = results[r]
        hops = ring_plan(r, world, 4 * world, causal, "contiguous")
        want_src = [h.src for h in hops if h.problems]
        want = [(c, s, 100 * c + s) for c in range(3) for s in want_src]
        assert seen == want
        # One pull per live hop after the first, the two receive slots alternating.
        pulls = [(s, g % 2) for g, s in enumerate(want_src) if g > 0]
        assert log == [e for _ in range(3) for e in [("pull", s, slot) for s, slot in pulls] + [("end",)]]


@pytest.mark.parametrize("world", [4, 6, 8])
@pytest.mark.parametrize("layout", ["zigzag", "contiguous"])
@pytest.mark.parametrize("causal", [False, True])
def test_merged_hops_cover_the_same_pairs(world, layout, causal):
    """A merged launch computes exactly the (query row, key) pairs of its member
    hops: every key row of the merged problems, read in the side-by-side
    receive buffer, is the key of the right shard at the right global position,
    no pair appears twice, and each problem keeps the kernel's limits (at most
    two key segments, a partially visible one last)."""
    seq = 32 * 2 * world
    for r in range(world):
        hops = ring_plan(r, world, seq, causal, layout)
        shard = seq // world
        srcsegs = {s: local_segments(s, world, seq, layout) for s in range(world)}
        groups = launch_groups(hops, shard)
        assert [h.src for m, _ in groups for h in m] == [h.src for h in hops if h.problems]
        for members, launched in groups:
            assert len(launched.problems) <= 4
            want, got = set(), []
            for h in members:
                for qr, ql, qp, keys in h.problems:
                    for kr, kl, kp in keys:
                        want |= {(qp + i, kp + j) for i in range(ql) for j in range(kl)}
            for qr, ql, qp, keys in launched.problems:
                assert 1 <= len(keys) <= 2
                if causal and len(keys) == 2:
                    assert keys[0][2] + keys[0][1] - 1 <= qp, "only the last key segment may be partial"
                for kr, kl, kp in keys:
                    j, row = divmod(kr, shard)
                    src = members[j].src
                    # rows [row, row + kl) of src's shard hold global positions [kp, kp + kl)
                    assert any(r0 <= row and row + kl <= r0 + n and kp == p0 + row - r0 for r0, n, p0 in srcsegs[src])
                    got += [(qp + i, kp + jj) for i in range(ql) for jj in range(kl)]
            assert len(got) == len(set(got)) and set(got) == want


def test_ring_exchange_protocol_with_merged_hops_over_gloo():
    """The same protocol when the transport pulls two shards into one buffer:
    on a 4-rank zigzag bf16 ring the middle (accumulate) hops of each rank go
    out as one launch whose K/V holds both hops' shards side by side, pulled
    with one pull_group; every hop's shard is still seen once per call, in hop
    order."""
    import socket

    import torch.multiprocessing as mp
    world = 4
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    pubs = [torch.zeros(2, 1, 1, 4, 2, dtype=torch.bfloat16).share_memory_() for _ in range(world)]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, pubs, True, results, "zigzag", torch.bfloat16, 2))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        seen, log = results[r]
        hops = ring_plan(r, world, 4 * world, True, "zigzag")
        want_src = [h.src for h in hops if h.problems]
        assert seen == [(c, s, 100 * c + s) for c in range(3) for s in want_src]
        groups = launch_groups(hops, 4)
        assert any(len(m) == 2 for m, _ in groups)
        pulls = []
        for g, (members, _) in enumerate(groups):
            if g:
                pulls.append(("pull", members[0].src, g % 2) if len(members) == 1 else
                             ("pull", tuple(h.src for h in members), g % 2))
        assert log == [e for _ in range(3) for e in pulls + [("end",)]]


@pytest.mark.parametrize("bh,per", [(16, 2), (64, 19), (1, 1), (2, 2), (3, 2), (5, 1), (7, 4), (4, 8), (16, 16),
                                    (100, 7)])
def test_host_chunks_cover_every_head_once(bh, per):
    """The host-input forward's chunks tile (batch x heads) in order, middle
    chunks at most `per`, the first and last at most about per / 2."""
    from algebraic_intelligence_b200.afa import _host_chunks
    ch = _host_chunks(bh, per)
    assert [i for a, b in ch for i in range(a, b)] == list(range(bh))
    assert all(0 < b - a <= per for a, b in ch)
    edge = max(1, per // 2)
    if bh > edge:
        assert ch[0][1] - ch[0][0] == edge


# ---------------------------------------------------------------------------
# The persistent kernel's work walk (afa_tc_sk_kernel, SkWalk in
# csrc/afa_tc_sm100.cu), restated: whole-item rounds, then an even split of the
# remaining key-tile iterations (accumulate hops), or whole items only in snake
# order (final output of short-pair prefills).
# ---------------------------------------------------------------------------
def _sk_before(prefix, nitems, nbh, j):
    pair, hh = divmod(j, nbh)
    base = nbh * prefix[pair]
    return base if pair >= nitems else base + hh * (prefix[pair + 1] - prefix[pair])


def _sk_walk(prefix, nitems, nbh, waves, snake, G, c):
    """The (bh, item, t0, t1) pieces CTA c of G computes, in order."""
    total = nbh * nitems
    out = []
    for k in range(waves):
        kc = G - 1 - c if (snake and k & 1) else c
        j = k * G + kc
        if j >= total:
            continue
        item, bh = divmod(j, nbh)
        n = prefix[item + 1] - prefix[item]
        if n > 0:
            out.append((bh, item, 0, n))
    if snake:
        return out
    j0 = waves * G
    i0 = _sk_before(prefix, nitems, nbh, j0)
    tail = _sk_before(prefix, nitems, nbh, total) - i0
    i, hi = i0 + tail * c // G, i0 + tail * (c + 1) // G
    while i < hi:
        lo, up = j0, total
        while up - lo > 1:
            mid = (lo + up) >> 1
            if _sk_before(prefix, nitems, nbh, mid) <= i:
                lo = mid
            else:
                up = mid
        item, bh = divmod(lo, nbh)
        t0 = i - _sk_before(prefix, nitems, nbh, lo)
        n = prefix[item + 1] - prefix[item]
        t1 = min(t0 + (hi - i), n)
        out.append((bh, item, t0, t1))
        i += t1 - t0
    return out


@pytest.mark.parametrize("snake", [False, True])
@pytest.mark.parametrize("seed", range(6))
def test_sk_walk_covers_every_key_tile_once(seed, snake):
    rng = np.random.default_rng(seed)
    nitems = int(rng.integers(1, 40))
    nbh = int(rng.integers(1, 70))
    lens = sorted((int(x) for x in rng.integers(1, 60, size=nitems)), reverse=True)
    prefix = np.concatenate([[0], np.cumsum(lens)]).tolist()
    items = nbh * nitems
    G = int(min(148, items if snake else max(1, nbh * prefix[-1] // 8)))
    waves = -(-items // G) if snake else items // G
    seen = {}
    for c in range(G):
        for bh, item, t0, t1 in _sk_walk(prefix, nitems, nbh, waves, snake, G, c):
            assert 0 <= t0 < t1 <= lens[item]
            if snake:
                assert (t0, t1) == (0, lens[item]), "final-output pieces are whole items"
            for t in range(t0, t1):
                assert (bh, item, t) not in seen
                seen[(bh, item, t)] = c
    assert len(seen) == nbh * prefix[-1]


def test_sk_walk_snake_balances_longest_first_lists():
    """Snake order over a longest-first list: every CTA's share of key tiles is
    within one item of the mean (config 3's causal pairs on 148 CTAs)."""
    nbh, npair = 64, 16
    lens = [2 * p + 2 for p in reversed(range(npair))]
    prefix = np.concatenate([[0], np.cumsum(lens)]).tolist()
    G = 148
    waves = -(-nbh * npair // G)
    work = [sum(t1 - t0 for _, _, t0, t1 in _sk_walk(prefix, npair, nbh, waves, True, G, c)) for c in range(G)]
    assert max(work) - min(work) <= max(lens)
