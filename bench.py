#!/usr/bin/env python
"""Benchmark of the B200 AFA hot path (one JSON line on rank 0).

Workload at every N (so per-N values compare like with like): BASELINE config 5,
ring AFA forward, B=1, H=16, L=65536, D=128, bf16, causal, the sequence
zigzag-sharded over N GPUs (one process per GPU; each hop pulls its K/V shard
from the owning GPU with the copy engines over NVLink, through CUDA IPC). At N=1 it is the single-GPU prefill forward of the whole sequence,
the largest single-GPU configuration of BASELINE.json.

  metric  "AFA fwd TFLOP/s": FLOPs = 4*B*H*D*L(L+1)/2 (QK^T and PV over the
          causal pairs; the octic map is not counted) / device time.
  value   whole-job throughput, inputs resident in HBM, max over ranks of the
          device time of exactly K steps (CUDA events, barrier + sync around).
  e2e     the same metric through the public API with host buffers: every step
          copies its Q/K/V shards from pinned host memory and the output back.

At N=1 the line also carries the other BASELINE configurations measured in the
same run (``sub``): config 3 (prefill L=4096, the 60%-of-peak target), config 2
(prefill L=2048 with K outliers), config 4 (decode, HBM GB/s), the backward
of config 3 and the AGO Q/K rotation at config 3's shape (HBM GB/s).

``--impl reference`` times the reference's CPU implementation of the path (the
float64 NumPy oracle of tests/reference_attention.py, restated in
oracle/afa_oracle.py) on a bounded sample of the same workload, with all host
cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

# Under torch.distributed.run (N > 1) each rank's NCCL communicator reports its
# rank and size when it is created (NCCL's INIT log lines; rank 0's JSON result
# is still one line of its own). NCCL reads these once, before torch is imported.
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    os.environ.setdefault("NCCL_DEBUG", "INFO")
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "AFA fwd TFLOP/s"
UNIT = "TFLOP/s"
RING = dict(B=1, H=16, L=65536, D=128)
CFG3 = dict(B=2, H=32, L=4096, D=128)
CFG2 = dict(B=4, H=16, L=2048, D=128)
DEC = dict(B=64, H=32, L=8192, D=128)
DEC_SMALL = dict(B=8, H=32, L=8192, D=128)  # profiling size (about 1 GB per input set)
SUB_IDLE_S = 0.5  # idle before each short sub-workload run


def causal_flops(B, H, L, D, **_):
    return 4.0 * B * H * D * L * (L + 1) / 2.0


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "of measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "of fallback"}


def load_traffic():
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices):
        self.indices = indices
        self.proc = None
        self.path = Path(f"/tmp/afa_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(i) for i in self.indices)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        try:
            self.path.unlink()
        except OSError:
            pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_index(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x for x in vis.split(",") if x.strip()]
        if local < len(ids) and ids[local].strip().isdigit():
            return int(ids[local])
    return local


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# timing
# ---------------------------------------------------------------------------
class KernelTimer:
    """CUDA-event pairs around each kernel launch, on the launching stream."""

    def __init__(self):
        self.pairs = []

    def around(self, fn):
        import torch
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        self.pairs.append((s, e))

    def mean_ms(self):
        return sum(s.elapsed_time(e) for s, e in self.pairs) / max(1, len(self.pairs))

    def count(self):
        return len(self.pairs)


def timed(step, steps, warmup, world):
    """Device time (ms) of exactly `steps` calls of step(i), max over ranks."""
    import torch
    for i in range(warmup):
        step(i, None)
    barrier(world)
    kt = KernelTimer()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step(i, kt)
    end.record()
    barrier(world)
    ms = start.elapsed_time(end)
    return max_over_ranks(ms, world), kt


def kernel_ms(launch, steps, warmup=3):
    """Mean device time (ms) of one launch: `steps` back-to-back launches
    through the C ABI with prepared arguments, bracketed by one CUDA event pair
    on the launching stream. For launches shorter than the host work of an API
    call (tens of microseconds of Python), events around each call would count
    the GPU idling while the host prepares the next one; here the stream stays
    busy, so the pair measures the kernels alone."""
    import torch
    for i in range(warmup):
        launch(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        launch(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def randn_bf16(shape, gen):
    import torch
    return torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).to(torch.bfloat16)


def ring_inputs(rank, world, seed):
    """This rank's zigzag shards of the global config-5 Q, K, V (generated per
    head on the device, identical on every rank)."""
    import torch
    from algebraic_intelligence_b200.ring import shard_sequence
    B, H, L, D = RING["B"], RING["H"], RING["L"], RING["D"]
    gen = torch.Generator(device="cuda").manual_seed(seed)
    out = []
    for _ in range(3):
        full = randn_bf16((B, H, L, D), gen)
        out.append(shard_sequence(full, rank, world, "zigzag") if world > 1 else full)
        del full
    return out


def run_ring(args, rank, world, peaks, traffic):
    import torch
    import algebraic_intelligence_b200 as afa
    from algebraic_intelligence_b200 import _lib
    from algebraic_intelligence_b200.afa import hop_forward
    from algebraic_intelligence_b200.ring import ring_plan

    sets = [ring_inputs(rank, world, seed) for seed in (0, 1)]  # 2 sets: > L2 between steps
    flops = causal_flops(**RING)
    hops = ring_plan(rank, world, RING["L"], True, "zigzag")
    if world > 1:
        from algebraic_intelligence_b200.ring import launch_groups
        launches_per_step = len(launch_groups(hops, RING["L"] // world))
    else:
        launches_per_step = 1

    if world == 1:
        def step(i, kt):
            q, k, v = sets[i % 2]
            f = lambda: afa.pallas_afa_forward(q, k, v, causal=True)  # noqa: E731
            kt.around(f) if kt else f()
    else:
        from algebraic_intelligence_b200.ring import get_exchange, ring_loop
        q0 = sets[0][0]
        b, h, s, d = q0.shape
        o_acc = torch.empty((b, h, s, d), dtype=torch.float32, device="cuda")
        d_acc = torch.empty((b, h, s), dtype=torch.float32, device="cuda")
        den = torch.empty((b, h, s, 1), dtype=torch.float32, device="cuda")
        out = torch.empty_like(q0)
        exchange = get_exchange(q0.shape, q0.dtype, q0.device)   # the one distributed_ring_afa uses
        phases = PhaseTimer()
        timed_exchange = TimedExchange(exchange, phases)

        def step(i, kt):
            q, k, v = sets[i % 2]

            def compute(hop, kk, vv):
                f = lambda: hop_forward(q, kk, vv, hop.problems, True, hop.mode, o_acc=o_acc,  # noqa: E731
                                        d_acc=d_acc, out=out, d_total=den, sink_omega=0.5)
                if kt is None:
                    f()
                    return
                name = {_lib.AFA_HOP_STORE: "hop0_store", _lib.AFA_HOP_FINALIZE: "hop_last_finalize"}.get(
                    hop.mode, "hop_accumulate")
                phases.around(name, lambda: kt.around(f))

            ring_loop(k, v, hops, compute, timed_exchange if kt is not None else exchange)

    ms, kt = timed(step, args.steps, args.warmup, world)
    value = flops * args.steps / (ms / 1e3) / 1e12
    launch_ms = kt.mean_ms()
    per_launch_flops = flops / world / launches_per_step
    achieved = per_launch_flops / (launch_ms / 1e3) / 1e12
    tr = traffic.get("ring_n1" if world == 1 else f"ring_n{world}")
    if tr is not None and world > 1:
        # The capture is of one accumulate hop; a launch here carries
        # live hops / launches of them on average (two middle hops merge), and
        # the bytes of a hop's K/V, Q and accumulators scale with its count.
        tr = tr * sum(1 for h in hops if h.problems) / launches_per_step
    res = {
        "value": value,
        "ms_per_step": ms / args.steps,
        "tok_per_s": RING["L"] * RING["B"] * args.steps / (ms / 1e3),
        # One attention kernel per launch (a hop, or two merged middle hops);
        # the last hop of a ring call (FINALIZE) also launches its divide pass
        # after the persistent accumulate kernel.
        "gpu_launches": kt.count() + (args.steps if world > 1 else 0),
        "roofline": {"bound": "tensor", "kernel": "afa_tc_fwd_kernel<128>" if world == 1 else
                     "afa_tc_fwd_kernel<128> (first hop) / afa_tc_sk_kernel<128> (other hops)", "achieved": achieved,
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "traffic": tr, "peak_source": peaks["source"] + " bf16_tflops (burst)",
                     "launch_ms": launch_ms, "flops_per_launch": per_launch_flops},
    }
    if world > 1:
        # Where a ring step's time goes, max over ranks (ms per step; per launch
        # for the hop kernels): the first hop's STORE kernel, the accumulate
        # launches (two merged hops each where launch_groups pairs them), the
        # last hop (accumulate + divide), the publish and the close (what the
        # compute stream waits for of the K/V publish and the two barriers).
        res["hop_breakdown"] = {k: max_over_ranks(v, world) for k, v in phases.summary(args.steps).items()}
        res["hop_breakdown"]["launches_per_step"] = launches_per_step
    del sets
    return res


class PhaseTimer:
    """CUDA-event pairs per named phase, on the current stream."""

    def __init__(self):
        self.pairs = {}

    def around(self, name, fn):
        import torch
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        r = fn()
        e.record()
        self.pairs.setdefault(name, []).append((s, e))
        return r

    def summary(self, steps):
        out = {}
        for name, pairs in sorted(self.pairs.items()):
            tot = sum(s.elapsed_time(e) for s, e in pairs)
            out[f"{name}_ms_per_step"] = tot / steps
            if name.startswith("hop"):
                out[f"{name}_ms_per_launch"] = tot / len(pairs)
        return out


class TimedExchange:
    """The ring's exchange with its publish and close phases timed on the
    compute stream (the publish copy and its barrier run on the exchange's side
    stream beside hop 0, so the publish phase shows only what the compute
    stream itself waits for)."""

    def __init__(self, ex, phases):
        self.ex, self.phases, self.rank = ex, phases, ex.rank
        self.max_group = getattr(ex, "max_group", 1)   # merged hops exactly as the untimed exchange runs them

    def publish(self, k, v):
        return self.phases.around("publish_copy_and_barrier", lambda: self.ex.publish(k, v))

    def pull(self, src, slot):
        return self.ex.pull(src, slot)

    def pull_group(self, srcs, slot):
        return self.ex.pull_group(srcs, slot)

    def ready(self, token):
        return self.ex.ready(token)

    def finish(self):
        self.phases.around("close_join_and_barrier", self.ex.finish)


def run_ring_e2e(args, rank, world):
    """Public API with host buffers. N=1: pinned host Q/K/V go straight into
    pallas_afa_forward, which returns the output in host memory; N>1: pinned
    host shards -> device -> distributed_ring_afa -> host."""
    import torch
    import algebraic_intelligence_b200 as afa
    sets = ring_inputs(rank, world, 0)
    host = [t.cpu().pin_memory() for t in sets]
    dev = [torch.empty_like(t) for t in sets]
    out_host = torch.empty_like(host[0]).pin_memory()
    del sets

    def step(i, kt):
        if world == 1:
            # Host tensors straight into the public API, which streams them
            # through the GPU in chunks, copies overlapping the kernels.
            afa.pallas_afa_forward(host[0], host[1], host[2], causal=True)
            return
        for d_, h_ in zip(dev, host):
            d_.copy_(h_, non_blocking=True)
        y = afa.distributed_ring_afa(dev[0], dev[1], dev[2], causal=True, num_devices=world, layout="zigzag")
        out_host.copy_(y, non_blocking=True)

    steps = max(2, min(args.steps, 5))
    ms, _ = timed(step, steps, 1, world)
    flops = causal_flops(**RING)
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_host.numel() * out_host.element_size()
    return {"value": flops * steps / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": ms / steps}


def run_ring_hop(args, peaks, world=8, rank=0, hop_index=1):
    """Profiling aid: one accumulate hop of the config-5 ring at `world` GPUs
    (rank `rank`, hop `hop_index`), timed on this GPU with the ring's shapes."""
    import torch
    from algebraic_intelligence_b200.afa import hop_forward
    from algebraic_intelligence_b200.ring import ring_plan
    B, H, L, D = RING["B"], RING["H"], RING["L"], RING["D"]
    s = L // world
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (randn_bf16((B, H, s, D), gen) for _ in range(3))
    o_acc = torch.zeros((B, H, s, D), dtype=torch.float32, device="cuda")
    d_acc = torch.zeros((B, H, s), dtype=torch.float32, device="cuda")
    hop = ring_plan(rank, world, L, True, "zigzag")[hop_index]
    flops = sum(4 * B * H * D * ql * sum(kl for _, kl, _ in segs) for _, ql, _, segs in hop.problems)

    def step(i, kt):
        f = lambda: hop_forward(q, k, v, hop.problems, True, hop.mode, o_acc=o_acc, d_acc=d_acc,  # noqa: E731
                                sink_omega=0.5)
        kt.around(f) if kt else f()

    ms, kt = timed(step, args.steps, max(args.warmup, 1), 1)
    achieved = flops / (kt.mean_ms() / 1e3) / 1e12
    return {"hop": f"rank {rank} hop {hop_index} of {world}", "mode": hop.mode, "flops_per_launch": flops,
            "launch_ms": kt.mean_ms(), "achieved_tflops": achieved, "frac": achieved / peaks["bf16_tflops"]}


def run_prefill(cfg, args, peaks, outliers=False):
    import torch
    import algebraic_intelligence_b200 as afa
    B, H, L, D = cfg["B"], cfg["H"], cfg["L"], cfg["D"]
    sets = []
    for seed in (0, 1):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        q, k, v = (randn_bf16((B, H, L, D), gen) for _ in range(3))
        if outliers:
            n = round(0.05 * L)
            for bi in range(B):
                for hi in range(H):
                    rows = torch.randperm(L, generator=torch.Generator().manual_seed(bi * H + hi))[:n]
                    k[bi, hi, rows.cuda()] += 8.0
        sets.append((q, k, v))
    flops = causal_flops(**cfg)

    def step(i, kt):
        q, k, v = sets[i % 2]
        f = lambda: afa.pallas_afa_forward(q, k, v, causal=True)  # noqa: E731
        kt.around(f) if kt else f()

    steps = max(args.steps, 10)
    ms, kt = timed(step, steps, max(args.warmup, 3), 1)
    from algebraic_intelligence_b200 import _lib
    lib = _lib.load()
    outs = [(torch.empty_like(q), torch.empty((B, H, L), dtype=torch.float32, device=q.device)) for q, _, _ in sets]
    stream = _lib.stream_ptr(torch.device("cuda", torch.cuda.current_device()))

    def launch(i):
        (q, k, v), (o, d) = sets[i % 2], outs[i % 2]
        _lib.check(lib.afa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), d.data_ptr(), B, H, L, D,
                               _lib.AFA_BF16, 0.5, 1, 0, stream), "afa_fwd")

    kms = kernel_ms(launch, steps)
    ach = flops / (kms / 1e3) / 1e12
    return {"value": flops * steps / (ms / 1e3) / 1e12, "unit": UNIT, "ms_per_step": ms / steps,
            "flops": flops, "api_call_ms": kt.mean_ms(), "kernel_ms": kms,
            "roofline": {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": ach / peaks["bf16_tflops"], "peak_source": peaks["source"] + " bf16_tflops"}}


def run_backward(cfg, args, peaks):
    """Backward of a prefill configuration (tiled_afa_backward): dq, dk, dv
    from q, k, v, the forward's out and d_total, and g_out. FLOPs count the
    five products of pallas_afa.py:500-510 over causal pairs, 10*B*H*D per pair
    (2.5x the forward); the kernels also recompute S and dP, which is not
    counted."""
    import torch
    import algebraic_intelligence_b200 as afa
    B, H, L, D = cfg["B"], cfg["H"], cfg["L"], cfg["D"]
    sets = []
    for seed in (0, 1):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        q, k, v, g = (randn_bf16((B, H, L, D), gen) for _ in range(4))
        out, den = afa.pallas_afa_forward(q, k, v, causal=True, return_denominator=True)
        sets.append((q, k, v, out, den, g))
    flops = 2.5 * causal_flops(**cfg)

    def step(i, kt):
        q, k, v, out, den, g = sets[i % 2]
        f = lambda: afa.tiled_afa_backward(q, k, v, out, den, g, causal=True)  # noqa: E731
        kt.around(f) if kt else f()

    steps = max(args.steps, 10)
    ms, kt = timed(step, steps, max(args.warmup, 3), 1)
    from algebraic_intelligence_b200 import _lib
    lib = _lib.load()
    need = lib.afa_bwd_workspace_bytes(B, H, L, D, _lib.AFA_BF16)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    grads = [tuple(torch.empty_like(q) for _ in range(3)) for q, *_ in sets]
    dens = [den.reshape(B, H, L).contiguous() for *_, den, _ in sets]
    stream = _lib.stream_ptr(torch.device("cuda", torch.cuda.current_device()))

    def launch(i):
        (q, k, v, out, _, g), den, (dq, dk, dv) = sets[i % 2], dens[i % 2], grads[i % 2]
        _lib.check(lib.afa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), den.data_ptr(),
                               g.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, L, D, _lib.AFA_BF16,
                               0.5, 1, 0, ws.data_ptr(), need, stream), "afa_bwd")

    kms = kernel_ms(launch, steps)
    ach = flops / (kms / 1e3) / 1e12
    return {"value": flops * steps / (ms / 1e3) / 1e12, "unit": UNIT, "ms_per_step": ms / steps,
            "flops": flops, "kernels_per_step": 3, "api_call_ms": kt.mean_ms(), "kernel_ms": kms,
            "roofline": {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": ach / peaks["bf16_tflops"], "peak_source": peaks["source"] + " bf16_tflops"}}


def run_ago(cfg, args, peaks):
    """AGO rotation of Q and K (apply_ago_rotations, the attention layer's Q/K
    prologue) at a prefill configuration's shape, bf16 with float32 tables:
    HBM-bound, bytes = read + write of both tensors."""
    import torch
    import algebraic_intelligence_b200 as afa
    B, H, L, D = cfg["B"], cfg["H"], cfg["L"], cfg["D"]
    rot = afa.build_cayley_rotary_matrix(D, L, dtype=torch.float32)
    sets = []
    for seed in (0, 1):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        sets.append(tuple(randn_bf16((B, H, L, D), gen) for _ in range(2)))
    nbytes = 4.0 * B * H * L * D * 2

    def step(i, kt):
        q, k = sets[i % 2]
        f = lambda: afa.apply_ago_rotations(q, k, rotary_params=rot, seq_axis=2)  # noqa: E731
        kt.around(f) if kt else f()

    steps = max(args.steps, 10)
    ms, kt = timed(step, steps, max(args.warmup, 3), 1)
    from algebraic_intelligence_b200 import _lib
    lib = _lib.load()
    c, s = rot.c.contiguous(), rot.s.contiguous()
    outs = [(torch.empty_like(q), torch.empty_like(k)) for q, k in sets]
    stream = _lib.stream_ptr(torch.device("cuda", torch.cuda.current_device()))
    code, tcode = _lib.dtype_code(torch.bfloat16), _lib.dtype_code(c.dtype)

    def launch(i):
        (q, k), (qo, ko) = sets[i % 2], outs[i % 2]
        _lib.check(lib.afa_ago_rotate(q.data_ptr(), k.data_ptr(), qo.data_ptr(), ko.data_ptr(), c.data_ptr(),
                                      s.data_ptr(), tcode, B * H * L, D, L, 1, code, stream), "afa_ago_rotate")

    kms = kernel_ms(launch, steps)
    ach = nbytes / (kms / 1e3) / 1e9
    return {"value": nbytes * steps / (ms / 1e3) / 1e9, "unit": "GB/s", "ms_per_step": ms / steps,
            "bytes": nbytes, "api_call_ms": kt.mean_ms(), "kernel_ms": kms,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": ach / peaks["hbm_gbs"], "peak_source": peaks["source"] + " hbm_gbs"}}


def run_decode(args, peaks, cfg=DEC):
    import torch
    import algebraic_intelligence_b200 as afa
    B, H, L, D = cfg["B"], cfg["H"], cfg["L"], cfg["D"]
    gen = torch.Generator(device="cuda").manual_seed(0)
    sets = []
    for _ in range(2):
        q = randn_bf16((B, H, D), gen)
        k = randn_bf16((B, H, L, D), gen)
        v = randn_bf16((B, H, L, D), gen)
        sets.append((q, k, v))
    nbytes = 2.0 * B * H * L * D * 2 + 2.0 * B * H * D * 2

    def step(i, kt):
        q, k, v = sets[i % 2]
        f = lambda: afa.afa_decode(q, k, v)  # noqa: E731
        kt.around(f) if kt else f()

    steps = max(args.steps, 10)
    ms, kt = timed(step, steps, max(args.warmup, 3), 1)
    kms = kt.mean_ms()
    ach = nbytes / (kms / 1e3) / 1e9
    return {"value": nbytes * steps / (ms / 1e3) / 1e9, "unit": "GB/s", "ms_per_step": ms / steps,
            "bytes": nbytes,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": ach / peaks["hbm_gbs"], "peak_source": peaks["source"] + " hbm_gbs"}}


# ---------------------------------------------------------------------------
# CPU side: the reference's float64 NumPy oracle on a bounded sample
# ---------------------------------------------------------------------------
def cpu_sample_inputs():
    """Head 0 of the config-5 problem, bf16-rounded values in float64."""
    import numpy as np
    import torch
    L, D = RING["L"], RING["D"]
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn((L, D), generator=g).to(torch.bfloat16).to(torch.float64).numpy() for _ in range(3))
    return np.ascontiguousarray(q), np.ascontiguousarray(k), np.ascontiguousarray(v)


def cpu_sample_step(qkv, rows):
    """Oracle forward of the given query rows of head 0 (causal); returns FLOPs."""
    from oracle import afa_oracle as orc
    q, k, v = qkv
    orc.afa_blocked(q, k, v, causal=True, rows=rows, block=64)
    return float(sum(4.0 * RING["D"] * (int(r) + 1) for r in rows))


def cpu_rows(i, n=64):
    import numpy as np
    L = RING["L"]
    base = (i * 7919) % (L - n)
    return np.arange(base, base + n)


def cpu_baseline(seconds=12.0):
    cores = os.cpu_count() or 1
    qkv = cpu_sample_inputs()
    cpu_sample_step(qkv, cpu_rows(0, 8))
    t0 = time.perf_counter()
    flops, i = 0.0, 0
    while time.perf_counter() - t0 < seconds:
        flops += cpu_sample_step(qkv, cpu_rows(i))
        i += 1
    dt = time.perf_counter() - t0
    return {"value": flops / dt / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"config 5 head 0, {i} blocks of 64 query rows (causal, all visible keys), "
                      f"{dt:.1f} s of float64 NumPy oracle (oracle/afa_oracle.py, restating "
                      f"tests/reference_attention.py), BLAS threads = {cores}"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    qkv = cpu_sample_inputs()
    for i in range(args.warmup):
        cpu_sample_step(qkv, cpu_rows(i, 16))
    t0 = time.perf_counter()
    flops = 0.0
    for i in range(args.steps):
        # Blocks 1, 2, ...: block 0 (the first 64 rows, which see almost no causal
        # keys) would make a one-step sample measure call overhead alone.
        flops += cpu_sample_step(qkv, cpu_rows(i + 1))
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": "config 5: AFA fwd B=1,H=16,L=65536,D=128 causal; each step a bounded sample "
                               "(64 query rows of head 0 against all their visible keys)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "64 query rows x all visible keys of head 0 per step, float64 NumPy oracle "
                                   "(oracle/afa_oracle.py restating tests/reference_attention.py)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="all", choices=["all", "ring", "ring8_hop", "prefill3", "prefill2", "backward3", "ago3",
                                                      "decode", "decode_small"],
                    help="profiling aid: run one workload only (N=1)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.warmup < 3 and args.workload == "all":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    rank, world, local = dist_setup(args.gpus)
    peaks = load_peaks()
    traffic = load_traffic()
    from algebraic_intelligence_b200 import _lib
    _lib.load()

    if args.workload != "all":
        fn = {"ring": lambda: run_ring(args, rank, world, peaks, traffic),
              "ring8_hop": lambda: run_ring_hop(args, peaks),
              "prefill3": lambda: run_prefill(CFG3, args, peaks),
              "prefill2": lambda: run_prefill(CFG2, args, peaks, outliers=True),
              "backward3": lambda: run_backward(CFG3, args, peaks),
              "ago3": lambda: run_ago(CFG3, args, peaks),
              "decode": lambda: run_decode(args, peaks),
              "decode_small": lambda: run_decode(args, peaks, DEC_SMALL)}[args.workload]
        res = fn()
        if rank == 0:
            print(json.dumps({"workload": args.workload, **res}), flush=True)
        return

    clocks = ClockSampler([physical_index(local)] if world == 1 else [physical_index(i) for i in range(world)])
    if rank == 0:
        clocks.start()
    ring = run_ring(args, rank, world, peaks, traffic)
    clk = clocks.stop() if rank == 0 else None
    e2e = run_ring_e2e(args, rank, world)
    sub = {}
    if world == 1:
        # Each of these short runs starts from an idle GPU (SUB_IDLE_S), not in
        # the power state the headline's long run at the power cap left behind.
        for name, fn in (("prefill_config3_L4096", lambda: run_prefill(CFG3, args, peaks)),
                         ("prefill_config2_L2048_outliers", lambda: run_prefill(CFG2, args, peaks, outliers=True)),
                         ("decode_config4", lambda: run_decode(args, peaks)),
                         ("backward_config3_L4096", lambda: run_backward(CFG3, args, peaks)),
                         ("ago_rotate_config3_shape", lambda: run_ago(CFG3, args, peaks))):
            torch.cuda.synchronize()
            time.sleep(SUB_IDLE_S)
            sub[name] = fn()
    status = _lib.device_status(torch.device("cuda", local))
    if rank == 0:
        line = {
            "metric": METRIC, "value": ring["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ring["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 5: ring AFA fwd B=1,H=16,L=65536,D=128 bf16 causal, "
                                   f"zigzag sequence sharding over {world} GPU(s)",
                       "global_batch": RING["B"], "seq_len": RING["L"], "heads": RING["H"], "head_dim": RING["D"],
                       "parallelism": f"ring{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2: two alternating input sets of "
                             f"{2 * 3 * RING['L'] * RING['H'] * RING['D'] * 2 // world / 1e6:.0f} MB per GPU"},
            "tok_per_s": ring["tok_per_s"],
            "gpu_launches": ring["gpu_launches"],
            "roofline": ring["roofline"],
            **({"hop_breakdown": ring["hop_breakdown"]} if "hop_breakdown" in ring else {}),
            "e2e": e2e,
            "clocks": clk,
            "device_status": status,
        }
        if sub:
            line["sub"] = sub
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
