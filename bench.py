"""Benchmark: StreamingLLM block-sparse attention on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload all|fwdbwd|fwd|decode|fx]

Headline (``value``): BASELINE config 2 -- sparse prefill forward+backward,
B=4, H=32, N=16384, D=128, bf16, S=4, W=2048, BM=BN=128 -- as kept-block
TFLOP/s (F_fwd = nnz * B * H * 4 * BM * BN * D; fwd+bwd = 3.5 * F_fwd).
The problem is fixed and its B*H = 128 (batch, head) units are split
contiguously across the N ranks (strong scaling, no collective on the data
path); ``value`` = the whole problem's FLOPs / max-over-ranks time.  After
the timed region O, dQ, dK, dV are all-gathered (NCCL) and compared bit for
bit with a single-GPU run on rank 0.  Secondary lines (``extra``): config 3
prefill forward (TFLOP/s), config 4 decode (KV GB/s over the 2.1517e9
visible K/V bytes per step), both split the same way, and config 5 (the FX
pass on an 8-layer Llama-style decoder, one GPU).

The K timed fwd+bwd steps are replays of the step captured once into a
CUDA graph (the same kernels; the host queues the whole timed region at
once, so a stalled host thread cannot idle the GPU); an eager timed pass of
the same step follows and is reported in ``extra.fwdbwd.eager_pass``.
``e2e`` runs the same step K times through the public API from pinned host
buffers (Q, K, V, dO host->device, O, dQ, dK, dV device->host, every step;
copies in, compute and copies out on three streams, two steps in flight) and
reports each stage's median device time.
``roofline`` uses the dominant kernel's device time per step, from CUDA
events recorded by libsbfa around each launch in a further eager timed pass
with the dQ GEMM serialised after one dK/dV pass (SBFA_BWD_GROUPS=1), so
each kernel's duration is its own; the same figure for the overlapped eager
pass is ``extra.fwdbwd.roofline_overlapped_pass``.
``--impl reference`` times the upstream eager masked-attention algorithm
(the CPU oracle port) on the host cores instead.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "graph-kernel-injection_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

CFG2 = dict(B=4, H=32, N=16384, D=128, S=4, W=2048, BM=128, BN=128, dtype=torch.bfloat16)
CFG3 = dict(B=1, H=32, N=131072, D=128, S=4, W=4096, BM=128, BN=128, dtype=torch.float16)
CFG4 = dict(B=64, H=32, N=100001, D=128, S=4, W=2048, BM=1, BN=64, dtype=torch.float16)
CFG5 = dict(B=2, N=32768, hidden=4096, layers=8, H=32, D=128, mlp=11008, vocab=32000, S=4,
            W=2048, BM=64, BN=64, dtype=torch.bfloat16)

GQA_GROUP = 4   # query heads per K/V head in the grouped-query decode line

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


class Dist:
    def __init__(self, want: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if want != self.world:
            raise SystemExit(f"--gpus {want} but WORLD_SIZE={self.world}")
        self.pg = None

    def init(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
        torch.cuda.set_device(self.local)

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        import shard
        return shard.max_over_ranks(x)

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"sbfa_clocks_{os.getpid()}.csv")

    def start(self):
        """Starts sampling every 50 ms and returns once the first sample is
        written, so that nvidia-smi's own start-up (seconds of host CPU and
        driver calls) is over before a timed region begins."""
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 3.0 and self.proc.poll() is None:
            self.fh.flush()
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)

    def stop(self, window=None):
        """Median SM clock, its maximum and the throttle reasons seen.  With
        `window` = (t0, t1) in host wall-clock seconds (the timed region),
        only the samples taken inside it count (the whole run when none
        fell inside, which `in_window` = false then says)."""
        if self.proc is None:
            return None
        return self._summary(window)

    def _summary(self, window):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[1]), float(parts[2]),
                             {nm for nm, val in zip(names, parts[3:7]) if val.lower() == "active"}))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        inside = rows
        if window is not None:
            inside = [r for r in rows if window[0] <= r[0] <= window[1]]
        in_window = window is not None and bool(inside)
        if not inside:
            inside = rows
        sm = sorted(r[1] for r in inside)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[2] for r in rows),
                "reasons": sorted(set().union(*(r[3] for r in inside))),
                "samples": len(sm), "in_window": in_window,
                "sm_mhz_min": sm[0]}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------


def kept_blocks(cfg) -> int:
    import sparse_triton_kernel as stk
    m = stk.make_streaming_mask(1 if cfg is CFG4 else cfg["N"], cfg["N"],
                                stk.StreamingMaskSpec(cfg["S"], cfg["W"]), cfg["BM"], cfg["BN"],
                                device="cuda")
    return int(m.sum().item()), m


def f_fwd(cfg, nnz: int) -> float:
    return float(nnz) * cfg["B"] * cfg["H"] * 4 * cfg["BM"] * cfg["BN"] * cfg["D"]


def decode_bytes(cfg) -> tuple:
    """(K+V visible bytes, q+o bytes) per decode step for the streaming rule."""
    qpos = cfg["N"] - 1
    vis = min(cfg["S"], qpos + 1) + (qpos + 1 - max(min(cfg["S"], qpos + 1), qpos - cfg["W"] + 1))
    es = torch.tensor([], dtype=cfg["dtype"]).element_size()
    kv = cfg["B"] * cfg["H"] * 2 * vis * cfg["D"] * es
    qo = cfg["B"] * cfg["H"] * 2 * cfg["D"] * es
    return kv, qo


# algorithmic FLOPs of one launch, as a multiple of F_fwd (bwd total 2.5 F_fwd:
# dK/dV kernel = S, dP, dV, dK; dQ kernel = dQ)
KERNEL_WORK = {"fwd": 1.0, "dkdv": 2.0, "dq": 0.5}


def kernel_kind(name: str):
    for kind in ("dkdv", "dq", "fwd"):
        if name.startswith(kind):
            return kind
    if name.startswith(("decode_split", "decode_gqa")):
        return "decode"
    return None


STEP_MS = []  # device time of each timed step of the last time_steps call (rank-local)
HOST_MS = []  # host time each of those steps took to enqueue (rank-local)
WINDOW = None  # host wall-clock (start, end) of that timed region


def time_steps(dist, step, steps: int, warmup: int):
    """Untimed warm-up, then `steps` steps bracketed by a barrier and a
    device synchronisation on both sides, timed with CUDA events on the
    launching stream; returns (max-over-ranks ms, our kernel launches,
    per-kernel device time).  An event after every step also records each
    step's own device time in STEP_MS, which shows whether a slow run had
    one stalled step or was slow throughout, and HOST_MS holds the host time
    each step took to enqueue (a device step much longer than its kernels
    with a long host step means the GPU waited for the host).  The garbage
    collector is paused over the timed steps."""
    global STEP_MS, HOST_MS, WINDOW
    import gc
    import sbfa_native as native
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    native.timing_read()  # discard warm-up records
    native.timing(True)
    n0 = native.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    host = [0.0] * (steps + 1)
    gc.collect()
    gc.disable()
    try:
        wall0 = time.time()
        start.record()
        host[0] = time.perf_counter()
        for i in range(steps):
            step()
            marks[i].record()
            host[i + 1] = time.perf_counter()
        end.record()
        torch.cuda.synchronize()
    finally:
        gc.enable()
    dist.barrier()
    native.timing(False)
    HOST_MS = [(host[i + 1] - host[i]) * 1e3 for i in range(steps)]
    WINDOW = (wall0, time.time())
    STEP_MS = [(start if i == 0 else marks[i - 1]).elapsed_time(marks[i]) for i in range(steps)]
    launches = native.launch_count() - n0
    ms = start.elapsed_time(end)
    per_kernel = native.timing_read()
    return dist.max(ms), launches, per_kernel


def graph_steps(dist, step, steps: int, warmup: int):
    """The step captured once into a CUDA graph, then `warmup` untimed and
    `steps` timed replays, bracketed like time_steps (barrier and device
    synchronisation on both sides, CUDA events on the launching stream, the
    max over ranks).  A replay is one host call, so the whole timed region is
    queued in about a millisecond and a stalled host thread (seen on these
    shared boxes for tens of ms at a time) cannot leave the GPU idle.  Returns
    None and the reason when the capture fails."""
    import sbfa_native as native
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = native.launch_count()
    try:
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            step()
    except Exception as exc:  # noqa: BLE001 - reported, the eager timing stands
        torch.cuda.synchronize()
        return None, f"capture failed: {str(exc).splitlines()[0][:160]}"
    per_step = native.launch_count() - n0
    for _ in range(max(warmup, 1)):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    host = [0.0] * (steps + 1)
    wall0 = time.time()
    start.record()
    host[0] = time.perf_counter()
    for i in range(steps):
        graph.replay()
        marks[i].record()
        host[i + 1] = time.perf_counter()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    wall1 = time.time()
    ms = start.elapsed_time(end)
    res = {"ms": dist.max(ms), "launches": per_step * steps, "window": (wall0, wall1),
           "step_ms": [(start if i == 0 else marks[i - 1]).elapsed_time(marks[i])
                       for i in range(steps)],
           "host_ms": [(host[i + 1] - host[i]) * 1e3 for i in range(steps)]}
    del graph
    torch.cuda.synchronize()
    return res, "ok"


def tensor_peak(pk, clocks):
    """(peak TFLOP/s, label) for a tensor-bound kernel: the burst figure
    (cuBLAS bf16 at full clock) while the SM clock sampled during the timed
    region stays within 10 % of its maximum, else the sustained one."""
    if clocks and clocks.get("sm_max_mhz") and clocks["sm_mhz"] < 0.9 * clocks["sm_max_mhz"]:
        return pk["bf16_tflops_sustained"], "sustained"
    return pk["bf16_tflops"], "burst"


def roofline(per_kernel, flops_fwd, pk, peak_src, steps, clocks=None, kv_bytes=None,
             workload="", scale_units=1.0):
    """Roofline of the dominant kernel over `steps` timed steps.  flops_fwd /
    kv_bytes are this rank's algorithmic work per step, and `achieved`
    divides the kernel's share of it by the kernel's device time per step
    (the sum of its launches: the backward launches dK/dV and the dQ GEMM
    once per group of (b, h) units when it overlaps them); `traffic` is the
    committed ncu DRAM byte count of the kernel's work in one full-size step,
    scaled by this rank's share of the (batch, head) units."""
    if not per_kernel:
        return None
    name, (tot, cnt) = max(per_kernel.items(), key=lambda kv: kv[1][0])
    kind = kernel_kind(name)
    avg_s = tot / steps / 1e3
    if kind == "decode":
        achieved = kv_bytes / avg_s / 1e9   # one split launch reads every visible K/V row once
        peak, which = pk["hbm_gbs"], "HBM copy"
        unit, bound = "GB/s", "hbm"
    elif kind in KERNEL_WORK:
        achieved = KERNEL_WORK[kind] * flops_fwd / avg_s / 1e12
        peak, which = tensor_peak(pk, clocks)
        unit, bound = "TFLOP/s", "tensor"
    else:
        return None
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as fh:
            t = json.load(fh).get(f"{name}@{workload}")
        traffic = None if t is None else int(round(t * scale_units))
    return {"kernel": name, "bound": bound, "achieved": round(achieved, 2), "peak": peak,
            "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_source": f"{peak_src} ({which})",
            "ms_per_step": round(tot / steps, 4), "avg_launch_ms": round(tot / cnt, 4),
            "launches": cnt,
            "kernel_share": {k: round(v[0] / sum(x[0] for x in per_kernel.values()), 4)
                             for k, v in per_kernel.items()}}


def executed_mma_flops(mask, cfg, units, dq_gemms=3):
    """Tensor-core FLOPs each kernel issues per step for `units` (batch,
    head) pairs, from the kept tiles of the plans the kernels walk (the
    forward's 256-row query-pair tiles visit the union of both tiles' kept
    key tiles; the recomputing dQ kernel issues S, dP and dQ, the dQ GEMM
    over stored dS only dQ), next to the algorithmic FLOPs of the same
    launch."""
    import sparse_triton_kernel as stk
    D, N, dt = cfg["D"], cfg["N"], cfg["dtype"]
    out = {}
    for kind, pass_id, gemms in (("fwd", 0, 2), ("dkdv", 2, 4), ("dq", 1, dq_gemms)):
        p = stk._plan_for(mask, pass_id, dt, D, N, N, cfg["BM"], cfg["BN"])
        tm, tn = p["tiles"]
        tiles = int(p["nnz"].item())
        out[kind] = gemms * 2.0 * tm * tn * D * tiles * units
    return out


def make_inputs(cfg, seed: int, n_q=None, local=None):
    """Seeded N(0,1) Q, K, V of a configuration (x0.5 for config 3); with
    `local` = (start, stop) only that range of the (batch, head) units, as a
    [1, stop - start, N, D] tensor."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    mul = 0.5 if cfg is CFG3 else 1.0
    nq = cfg["N"] if n_q is None else n_q
    B, H = (cfg["B"], cfg["H"]) if local is None else (1, local[1] - local[0])
    q = torch.randn(B, H, nq, cfg["D"], generator=g, device=dev, dtype=cfg["dtype"])
    k = torch.randn(B, H, cfg["N"], cfg["D"], generator=g, device=dev, dtype=cfg["dtype"])
    v = torch.randn(B, H, cfg["N"], cfg["D"], generator=g, device=dev, dtype=cfg["dtype"])
    if mul != 1.0:
        for t in (q, k, v):
            t.mul_(mul)
    return q, k, v


def e2e_pipelined(dist, stk, mask, kw, host_in, dev_in, out_h, steps: int, warmup: int):
    """Milliseconds for `steps` end-to-end fwd+bwd steps (max over ranks):
    copy-in on one stream, compute on the current stream, copy-out on a
    third, with events ordering the reuse of the two buffer sets.  Also
    returns the median device time of each stage over the timed steps (rank
    0's), which shows which of the three bounds the pipeline.  The garbage
    collector is paused over the timed steps."""
    import gc
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def run(n, start_ev, stages=None):
        for i in range(n):
            b = i % 2
            st = None if stages is None else [torch.cuda.Event(enable_timing=True)
                                              for _ in range(6)]
            with torch.cuda.stream(s_in):
                s_in.wait_event(start_ev)
                if i >= 2:
                    s_in.wait_event(ev_comp[b])  # step i-2 has finished reading dev_in[b]
                if st:
                    st[0].record(s_in)
                for d, h in zip(dev_in[b], host_in):
                    d.copy_(h, non_blocking=True)
                if st:
                    st[1].record(s_in)
                ev_in[b].record(s_in)
            comp.wait_event(ev_in[b])
            if st:
                st[2].record(comp)
            qd, kd, vd, dod = dev_in[b]
            for t in (qd, kd, vd):
                t.requires_grad_(True)
                t.grad = None
            o = stk.block_sparse_attention(qd, kd, vd, mask, **kw)
            o.backward(dod)
            outs = (o.detach(), qd.grad, kd.grad, vd.grad)
            if st:
                st[3].record(comp)
            ev_comp[b].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp[b])
                if st:
                    st[4].record(s_out)
                for h, d in zip(out_h[b], outs):
                    h.copy_(d, non_blocking=True)
                    d.record_stream(s_out)
                if st:
                    st[5].record(s_out)
                ev_out[b].record(s_out)
            if st:
                stages.append(st)
            for t in (qd, kd, vd):
                t.grad = None
                t.requires_grad_(False)
        comp.wait_event(ev_out[(n - 1) % 2])
        if n >= 2:
            comp.wait_event(ev_out[(n - 2) % 2])

    ev0 = torch.cuda.Event()
    ev0.record(comp)
    run(warmup, ev0)
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stages = []
    gc.collect()
    gc.disable()
    try:
        start.record(comp)
        run(steps, start, stages)
        end.record(comp)
        torch.cuda.synchronize()
    finally:
        gc.enable()
    dist.barrier()

    def med(a, b):
        return round(statistics.median(st[a].elapsed_time(st[b]) for st in stages), 3)

    stage_ms = {"h2d": med(0, 1), "compute": med(2, 3), "d2h": med(4, 5)}
    return dist.max(start.elapsed_time(end)), stage_ms


def local_units(dist, cfg):
    """This rank's contiguous share [start, stop) of the B*H (batch, head)
    units of a configuration (the whole range on one GPU)."""
    import shard
    return shard.shard_units(cfg["B"] * cfg["H"], dist.world, dist.rank)


def gather_units(dist, t, start, stop, units):
    """All ranks' [1, n, ...] slices of a (batch, head)-sharded tensor,
    reassembled on every rank as [units, ...] (NCCL all_gather; shards are
    padded to the largest one)."""
    import shard
    sizes = [b - a for a, b in (shard.shard_units(units, dist.world, r)
                                for r in range(dist.world))]
    cap = max(sizes)
    flat = t.reshape(stop - start, *t.shape[2:])
    if dist.world == 1:
        return flat
    import torch.distributed as tdist
    pad = torch.zeros((cap,) + tuple(flat.shape[1:]), dtype=flat.dtype, device=flat.device)
    pad[: stop - start] = flat
    out = torch.empty((dist.world * cap,) + tuple(flat.shape[1:]), dtype=flat.dtype,
                      device=flat.device)
    tdist.all_gather_into_tensor(out, pad)
    return torch.cat([out[r * cap: r * cap + n] for r, n in enumerate(sizes)])


def bench_fwdbwd(dist, args, pk, src):
    """Config 2 fwd+bwd.  The global problem is fixed (B=4, H=32: 128
    (batch, head) units); each rank takes a contiguous share of the units
    (strong scaling) and reads it as a [1, units, N, D] view, with no
    collective on the data path.  After the timed region every rank's O, dQ,
    dK, dV are all-gathered (NCCL) and rank 0 compares them bit for bit with
    its own single-GPU run of the whole problem on the same inputs."""
    import shard
    import sparse_triton_kernel as stk
    cfg = CFG2
    nnz, mask = kept_blocks(cfg)
    F = f_fwd(cfg, nnz)                       # the whole problem
    units = cfg["B"] * cfg["H"]
    start, stop = local_units(dist, cfg)
    F_local = F * (stop - start) / units
    q_full, k_full, v_full = make_inputs(cfg, 0)
    g1 = torch.Generator(device="cuda").manual_seed(1)
    do_full = torch.randn(q_full.shape, generator=g1, device="cuda", dtype=cfg["dtype"])
    q, k, v, do = (shard.bh_slice(t, start, stop).clone()
                   for t in (q_full, k_full, v_full, do_full))
    if dist.rank != 0:
        del q_full, k_full, v_full, do_full
    for t in (q, k, v):
        t.requires_grad_(True)
    kw = dict(block_m=cfg["BM"], block_n=cfg["BN"], is_causal=True, sink_size=cfg["S"],
              window_size=cfg["W"])

    def step():
        for t in (q, k, v):
            t.grad = None
        o = stk.block_sparse_attention(q, k, v, mask, **kw)
        o.backward(do)
        return o

    # headline: the step replayed from a CUDA graph; per-kernel device
    # times (the roofline) from an eager timed pass of the same step
    clocks = ClockSampler(dist.local)
    clocks.start()
    gres, gwhy = graph_steps(dist, step, args.steps, args.warmup)
    clk = clocks.stop(gres["window"] if gres is not None else None)
    eclocks = ClockSampler(dist.local)
    eclocks.start()
    e_ms, e_launches, per_kernel = time_steps(dist, step, args.steps, args.warmup)
    eclk = eclocks.stop(WINDOW)
    eager = {"ms_per_step": round(e_ms / args.steps, 3), "launches": e_launches,
             "step_ms_rank0": [round(x, 3) for x in STEP_MS],
             "host_enqueue_ms_rank0": [round(x, 3) for x in HOST_MS], "clocks": eclk}
    if gres is None:
        ms, launches, clk = e_ms, e_launches, eclk
        step_ms, host_ms = list(STEP_MS), list(HOST_MS)
    else:
        ms, launches = gres["ms"], gres["launches"]
        step_ms, host_ms = gres["step_ms"], gres["host_ms"]
    value = 3.5 * F * args.steps / (ms / 1e3) / 1e12
    # roofline pass: with the dQ GEMM overlapped, dK/dV and dQ share the SMs
    # and each one's CUDA-event duration includes the other's; this eager
    # pass runs one dK/dV pass and then the dQ GEMM, so each duration is the
    # kernel's own (the shares then compare with ncu's serialised launches)
    old_groups = os.environ.get("SBFA_BWD_GROUPS")
    os.environ["SBFA_BWD_GROUPS"] = "1"
    try:
        _, _, per_kernel_iso = time_steps(dist, step, args.steps, args.warmup)
    finally:
        if old_groups is None:
            os.environ.pop("SBFA_BWD_GROUPS", None)
        else:
            os.environ["SBFA_BWD_GROUPS"] = old_groups

    # verification (outside the timed region)
    o = step()
    torch.cuda.synchronize()
    got = [gather_units(dist, x.detach(), start, stop, units)
           for x in (o, q.grad, k.grad, v.grad)]
    verify = None
    if dist.rank == 0:
        qf, kf, vf = (t.clone().requires_grad_(True) for t in (q_full, k_full, v_full))
        of = stk.block_sparse_attention(qf, kf, vf, mask, **kw)
        of.backward(do_full)
        ref = [x.detach().reshape(units, *x.shape[2:]) for x in (of, qf.grad, kf.grad, vf.grad)]
        same = [bool(torch.equal(a, b)) for a, b in zip(got, ref)]
        finite = all(bool(torch.isfinite(a).all()) for a in got)
        verify = {"gathered": "O, dQ, dK, dV of all ranks (NCCL all_gather)" if dist.world > 1
                  else "O, dQ, dK, dV (one rank)",
                  "bitwise_equal_to_1gpu_run": dict(zip(("o", "dq", "dk", "dv"), same)),
                  "finite": finite}
        del qf, kf, vf, of, ref, q_full, k_full, v_full, do_full
    del got

    # e2e through the public API from pinned host memory: every step copies its
    # inputs (Q, K, V, dO) host->device and its results (O, dQ, dK, dV)
    # device->host.  Copies in, compute and copies out run on three streams,
    # two steps deep (device input buffers and host output buffers alternate),
    # so step s+1's inputs and step s-1's results move while step s computes.
    hq, hk, hv, hdo = (t.detach().to("cpu").pin_memory() for t in (q, k, v, do))
    host_in = (hq, hk, hv, hdo)
    out_h = [[torch.empty(q.shape, dtype=cfg["dtype"]).pin_memory() for _ in range(4)]
             for _ in range(2)]
    dev_in = [[torch.empty_like(t) for t in (q, k, v, do)] for _ in range(2)]
    e_steps = max(2, args.steps)
    e_ms, e_stages = float("nan"), None
    if not args.no_e2e:
        e_ms, e_stages = e2e_pipelined(dist, stk, mask, kw, host_in, dev_in, out_h, e_steps,
                                       warmup=2)
    bytes_h2d = sum(t.numel() * t.element_size() for t in host_in)
    bytes_d2h = sum(t.numel() * t.element_size() for t in out_h[0])
    e2e = None if args.no_e2e else {
        "value": round(3.5 * F * e_steps / (e_ms / 1e3) / 1e12, 3),
        "unit": "TFLOP/s", "h2d_bytes_per_step": bytes_h2d * dist.world,
        "d2h_bytes_per_step": bytes_d2h * dist.world,
        "ms_per_step": round(e_ms / e_steps, 3), "steps": e_steps,
        "stage_ms_median_rank0": e_stages,
        "pipeline": "copy-in / compute / copy-out on three streams, two steps in flight"}
    if e2e is not None:
        e2e["copies"] = copy_peaks(dist, host_in, dev_in[0], out_h[0], e_ms / e_steps)
    del dev_in, hq, hk, hv, hdo, host_in, out_h
    rl_ovl = roofline(per_kernel, F_local, pk, src, args.steps, clocks=clk, workload="cfg2",
                      scale_units=(stop - start) / units)
    rl = roofline(per_kernel_iso, F_local, pk, src, args.steps, clocks=clk, workload="cfg2",
                  scale_units=(stop - start) / units)
    if rl is not None:
        rl["timed_as"] = ("eager pass with the dQ GEMM after one dK/dV pass "
                          "(SBFA_BWD_GROUPS=1), so each kernel's duration is its own")
    res = dict(value=value, ms=ms, launches=launches, clocks=clk, e2e=e2e, roofline=rl,
               roofline_overlapped=rl_ovl, per_kernel_iso=per_kernel_iso,
               nnz=nnz, flops_fwd=F, verify=verify, per_kernel=per_kernel, step_ms=step_ms,
               host_ms=host_ms, eager=eager,
               timing=("CUDA-graph replays of the captured fwd+bwd step" if gres is not None
                       else f"eager steps ({gwhy})"),
               units=(start, stop, units))
    del q, k, v, do
    torch.cuda.empty_cache()
    if dist.world > 1 and not args.no_weak:
        res["weak"] = bench_fwdbwd_weak(dist, args, F)
    return res


def copy_peaks(dist, host_in, dev_bufs, host_out, step_ms):
    """Pinned host<->device copy bandwidth of this rank's e2e tensors, each
    direction alone and both at once (the pipelined step overlaps them), and
    the copy-bound floor of one e2e step it implies (max over ranks)."""
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    nbytes_in = sum(t.numel() * t.element_size() for t in host_in)
    nbytes_out = sum(t.numel() * t.element_size() for t in host_out)

    def timed(h2d: bool, d2h: bool, reps: int = 2) -> float:
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for st in (s_in, s_out):
            st.wait_event(a)
        for _ in range(reps):
            if h2d:
                with torch.cuda.stream(s_in):
                    for d, h in zip(dev_bufs, host_in):
                        d.copy_(h, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s_out):
                    for h, d in zip(host_out, dev_bufs):
                        h.copy_(d, non_blocking=True)
        cur = torch.cuda.current_stream()
        for st in (s_in, s_out):
            cur.wait_stream(st)
        b.record()
        torch.cuda.synchronize()
        return dist.max(a.elapsed_time(b) / reps)

    h2d_ms, d2h_ms, both_ms = timed(True, False), timed(False, True), timed(True, True)
    return {"h2d_gbs": round(nbytes_in / h2d_ms / 1e6, 1),
            "d2h_gbs": round(nbytes_out / d2h_ms / 1e6, 1),
            "both_directions_ms": round(both_ms, 3),
            "copy_bound_fraction": round(both_ms / step_ms, 3),
            "note": "pinned copies of the step's own tensors, per rank; copy_bound_fraction ="
                    " both-direction copy time / e2e step time"}


def bench_fwdbwd_weak(dist, args, F):
    """Weak scaling for reference: every rank runs the whole config-2 batch
    (the job's batch is 4 * N); value = all ranks' FLOPs / max time, timed
    like the headline (CUDA-graph replays, eager steps if the capture
    fails)."""
    import sparse_triton_kernel as stk
    cfg = CFG2
    _, mask = kept_blocks(cfg)
    q, k, v = make_inputs(cfg, dist.rank)
    g1 = torch.Generator(device="cuda").manual_seed(1000 + dist.rank)
    do = torch.randn(q.shape, generator=g1, device="cuda", dtype=cfg["dtype"])
    for t in (q, k, v):
        t.requires_grad_(True)
    kw = dict(block_m=cfg["BM"], block_n=cfg["BN"], is_causal=True, sink_size=cfg["S"],
              window_size=cfg["W"])

    def step():
        for t in (q, k, v):
            t.grad = None
        stk.block_sparse_attention(q, k, v, mask, **kw).backward(do)

    steps = max(2, args.steps)
    gres, gwhy = graph_steps(dist, step, steps, args.warmup)
    if gres is not None:
        ms, timed = gres["ms"], "CUDA-graph replays of the captured fwd+bwd step"
    else:
        ms, _, _ = time_steps(dist, step, steps, args.warmup)
        timed = f"eager steps ({gwhy})"
    del q, k, v, do
    torch.cuda.empty_cache()
    return {"value": round(3.5 * F * dist.world * steps / (ms / 1e3) / 1e12, 3),
            "unit": "TFLOP/s", "ms_per_step": round(ms / steps, 3), "global_batch": 4 * dist.world,
            "scaling": "weak", "timed_as": timed}


def bench_fwd(dist, args, pk, src):
    """Config 3 prefill forward; the 32 (batch, head) units are split across
    ranks like config 2's."""
    import sparse_triton_kernel as stk
    cfg = CFG3
    nnz, mask = kept_blocks(cfg)
    F = f_fwd(cfg, nnz)
    start, stop = local_units(dist, cfg)
    units = cfg["B"] * cfg["H"]
    q, k, v = make_inputs(cfg, dist.rank, local=(start, stop))
    kw = dict(block_m=cfg["BM"], block_n=cfg["BN"], is_causal=True, sink_size=cfg["S"],
              window_size=cfg["W"])

    def step():
        with torch.no_grad():
            return stk.block_sparse_attention(q, k, v, mask, **kw)

    steps = max(2, args.steps)
    clocks = ClockSampler(dist.local)
    clocks.start()
    ms, launches, per_kernel = time_steps(dist, step, steps, args.warmup)
    clk = clocks.stop(WINDOW)
    value = F * steps / (ms / 1e3) / 1e12
    share = (stop - start) / units
    rl = roofline(per_kernel, F * share, pk, src, steps, clocks=clk, workload="cfg3",
                  scale_units=share)
    del q, k, v
    torch.cuda.empty_cache()
    return dict(value=value, ms=ms / steps, roofline=rl, nnz=nnz, launches=launches, clocks=clk,
                units=(start, stop, units))


def bench_decode(dist, args, pk, src):
    """Config 4 decode over a full 100001-token cache, then over a
    StreamingLLM ring cache; the 2048 (batch, head) units are split across
    ranks."""
    import sparse_triton_kernel as stk
    cfg = CFG4
    _, mask = kept_blocks(cfg)
    start, stop = local_units(dist, cfg)
    units = cfg["B"] * cfg["H"]
    share = (stop - start) / units
    # the ring cache of the second measurement is allocated before the full
    # cache, on an empty device (as a serving process would hold it)
    from streaming_kv_cache import StreamingKVCache
    cache = StreamingKVCache(1, stop - start, cfg["D"], cfg["S"], cfg["W"], dtype=cfg["dtype"])
    # grouped-query variant: the same query heads over GQA_GROUP times fewer
    # K/V heads (allocated up front too, before the full cache)
    n_loc = stop - start
    gq = GQA_GROUP if n_loc % GQA_GROUP == 0 else 1
    gen = torch.Generator(device="cuda").manual_seed(99)
    k_g = torch.randn(1, n_loc // gq, cfg["N"], cfg["D"], generator=gen, device="cuda",
                      dtype=cfg["dtype"])
    v_g = torch.randn_like(k_g)
    q, k, v = make_inputs(cfg, dist.rank, n_q=1, local=(start, stop))
    kv_bytes, qo_bytes = decode_bytes(cfg)        # the whole problem
    kw = dict(block_m=cfg["BM"], block_n=cfg["BN"], is_causal=True, sink_size=cfg["S"],
              window_size=cfg["W"])

    def step():
        with torch.no_grad():
            return stk.block_sparse_attention(q, k, v, mask, **kw)

    steps = max(5, args.steps * 5)
    ms, launches, per_kernel = time_steps(dist, step, steps, args.warmup)
    value = kv_bytes * steps / (ms / 1e3) / 1e9
    rl = roofline(per_kernel, 0.0, pk, src, steps, kv_bytes=kv_bytes * share, workload="cfg4",
                  scale_units=share)

    # the same decode over a StreamingLLM ring cache holding sink + window rows
    # (timed before the full cache is freed: a large free is followed by the
    # driver clearing that memory, which competes for HBM bandwidth for a while)
    cache.append(k, v)
    full_bytes = 2 * k.numel() * k.element_size()

    def ring_step():
        return cache.attend(q)

    r_ms, r_launches, r_per_kernel = time_steps(dist, ring_step, steps, args.warmup)

    def gqa_step():
        with torch.no_grad():
            return stk.block_sparse_attention(q, k_g, v_g, mask, **kw)

    g_ms, g_launches, g_per_kernel = time_steps(dist, gqa_step, steps, args.warmup)
    g_bytes = kv_bytes / gq        # each K/V head's visible rows, read once for its group
    gqa = {"value": round(g_bytes * steps / (g_ms / 1e3) / 1e9, 2), "unit": "GB/s",
           "ms_per_step": round(g_ms / steps, 4), "kv_heads_per_query_heads": f"1/{gq}",
           "kv_bytes_per_step": int(g_bytes),
           "roofline": roofline(g_per_kernel, 0.0, pk, src, steps, kv_bytes=g_bytes * share,
                                workload=f"cfg4_gqa{gq}", scale_units=share),
           "gpu_launches": g_launches,
           "config": f"config 4 geometry with {CFG4['H'] // gq} K/V heads for {CFG4['H']} "
                     "query heads (grouped-query attention)"}
    del k_g, v_g
    ring = {"value": round(kv_bytes * steps / (r_ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(r_ms / steps, 4), "cache_bytes": cache.memory_bytes,
            "full_cache_bytes": full_bytes,
            "memory_ratio": round(full_bytes / cache.memory_bytes, 2),
            "roofline": roofline(r_per_kernel, 0.0, pk, src, steps, kv_bytes=kv_bytes * share,
                                 workload="cfg4_ring", scale_units=share),
            "gpu_launches": r_launches}
    del q, k, v, cache
    torch.cuda.empty_cache()
    return dict(value=value, ms=ms / steps, roofline=rl, kv_bytes=kv_bytes, qo_bytes=qo_bytes,
                launches=launches, ring=ring, gqa=gqa, units=(start, stop, units))


def bench_fx(dist, args, pk, src):
    """Config 5: the Llama-style decoder rewritten by the FX pass, one
    forward + backward step (loss = cross entropy on random targets; no
    optimizer step, as the config specifies).  Reports tokens/s of the whole
    step and the share of the step spent in this library's kernels."""
    import torch.nn.functional as F  # noqa: N812

    import sparse_triton_kernel as stk
    from fx_compiler_pass import BlockSparseAttentionInjector, InjectionConfig, LlamaStyleDecoder
    cfg = dict(CFG5)
    if args.fx_layers > 0:
        cfg["layers"] = args.fx_layers
    torch.manual_seed(1234 + dist.rank)
    model = LlamaStyleDecoder(vocab=cfg["vocab"], hidden=cfg["hidden"], n_layers=cfg["layers"],
                              n_heads=cfg["H"], mlp=cfg["mlp"], max_seq=cfg["N"],
                              device="cuda", dtype=cfg["dtype"])
    icfg = InjectionConfig(seq_len_q=cfg["N"], seq_len_kv=cfg["N"], head_dim=cfg["D"],
                           streaming=stk.StreamingMaskSpec(cfg["S"], cfg["W"]),
                           block_m=cfg["BM"], block_n=cfg["BN"])
    gm = BlockSparseAttentionInjector(icfg).transform(model).to("cuda")
    n_inj = sum(1 for n in gm.graph.nodes
                if n.op == "call_module" and str(n.target).startswith("_triton_attn_"))
    g = torch.Generator(device="cuda").manual_seed(dist.rank)
    ids = torch.randint(0, cfg["vocab"], (cfg["B"], cfg["N"]), generator=g, device="cuda")
    tgt = torch.randint(0, cfg["vocab"], (cfg["B"], cfg["N"]), generator=g, device="cuda")
    params = list(model.parameters())

    def step():
        for p in params:
            p.grad = None
        logits = gm(ids)
        loss = F.cross_entropy(logits.view(-1, cfg["vocab"]).float(), tgt.view(-1))
        loss.backward()
        return loss

    steps = max(2, min(args.steps, 3))
    ms, launches, per_kernel = time_steps(dist, step, steps, args.warmup)
    loss = float(step().item())
    ours_ms = sum(v[0] for v in per_kernel.values())
    nnz = int(stk.make_streaming_mask(cfg["N"], cfg["N"], stk.StreamingMaskSpec(cfg["S"], cfg["W"]),
                                      cfg["BM"], cfg["BN"], device="cuda").sum().item())
    attn_flops = 3.5 * nnz * cfg["B"] * cfg["H"] * 4 * cfg["BM"] * cfg["BN"] * cfg["D"] * \
        cfg["layers"]
    n_params = sum(p.numel() for p in params)
    tokens = cfg["B"] * cfg["N"]
    res = {"tokens_per_s": round(tokens * dist.world * steps / (ms / 1e3), 1),
           "ms_per_step": round(ms / steps, 2), "layers": cfg["layers"],
           "injected_modules": n_inj, "kept_blocks": nnz, "loss": round(loss, 4),
           "attention_ms_per_step": round(ours_ms / steps, 2),
           "attention_share": round(ours_ms / ms, 4),
           "attention_tflops": round(attn_flops * steps / (ours_ms / 1e3) / 1e12, 1),
           "model_tflops_est": round((6 * n_params * tokens + attn_flops) * steps /
                                     (ms / 1e3) / 1e12, 1),
           "params": n_params, "gpu_launches": launches,
           "per_kernel_ms": {k: round(v[0] / steps, 3) for k, v in per_kernel.items()},
           "config": "8-layer Llama-style decoder (hidden 4096, 32 heads, D=128, SwiGLU "
                     "11008, RMSNorm, RoPE), bf16 random init, B=2 N=32768, SDPA(is_causal) "
                     f"rewritten by the FX pass, S=4 W=2048 BM=BN={cfg['BM']}"}
    del gm, model, params, ids, tgt
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# CPU baseline (upstream eager masked attention, oracle port)
# ---------------------------------------------------------------------------


def cpu_baseline_fwdbwd(budget_s: float = 20.0):
    """Eager fwd+bwd of one (batch, head) slice of config 2 on the host:
    the bottom-right 1024 query rows against all 16384 keys (fp32), repeated
    while the budget lasts, extrapolated x16 rows x128 slices."""
    from oracle import streaming_oracle as orc
    cfg = CFG2
    rows = 1024
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 1, rows, cfg["D"], generator=g)
    k = torch.randn(1, 1, cfg["N"], cfg["D"], generator=g)
    v = torch.randn(1, 1, cfg["N"], cfg["D"], generator=g)
    do = torch.randn(1, 1, rows, cfg["D"], generator=g)
    mask = orc.make_streaming_mask(rows, cfg["N"], cfg["S"], cfg["W"], cfg["BM"], cfg["BN"])
    kw = dict(block_m=cfg["BM"], block_n=cfg["BN"], is_causal=True, sink_size=cfg["S"],
              window_size=cfg["W"])
    orc.attention_forward_backward(q, k, v, do, mask, **kw)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        orc.attention_forward_backward(q, k, v, do, mask, **kw)
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 20:
            break
    per = (time.perf_counter() - t0) / n
    full_step_s = per * (cfg["N"] / rows) * cfg["B"] * cfg["H"]
    nnz = int(orc.make_streaming_mask(cfg["N"], cfg["N"], cfg["S"], cfg["W"], cfg["BM"],
                                      cfg["BN"]).sum())
    flops = 3.5 * f_fwd(cfg, nnz)
    return {"value": round(flops / full_step_s / 1e12, 6), "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"1 of 128 (b,h) slices; bottom-right {rows} of {cfg['N']} query rows x "
                      f"{cfg['N']} keys; fp32 eager fwd+bwd (torch autograd), {n} reps of "
                      f"{per:.3f} s; extrapolated x{cfg['N'] // rows} rows x128 slices",
            "seconds_per_full_step": round(full_step_s, 2)}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------


def base_line(args, world):
    units = CFG2["B"] * CFG2["H"]
    return {"metric": "kept-block attn TFLOP/s fwd+bwd", "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v/dO, BASELINE config 2 shapes)",
            "config": {"workload": "cfg2 sparse prefill fwd+bwd: B=4 H=32 N=16384 D=128 bf16 "
                                   "S=4 W=2048 BM=BN=128 (whole problem, split across GPUs)",
                       "global_batch": CFG2["B"], "seq_len": 16384, "heads": CFG2["H"],
                       "head_dim": 128,
                       "parallelism": f"(batch,head) shards: {units} units over {world} GPU(s)",
                       "l2": "inputs exceed L2 (537 MB per tensor at 1 GPU; "
                             f"{537 // world} MB per GPU at {world}); no flush"}}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    budget = max(10.0, min(60.0, 6.0 * args.steps))
    cb = cpu_baseline_fwdbwd(budget_s=budget)
    line = base_line(args, world)
    line.update({"impl": "reference", "value": cb["value"],
                 "ms_per_step": round(cb["seconds_per_full_step"] * 1e3, 1),
                 "dtype": "f32 (host eager)", "cpu_baseline": cb,
                 "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}, "gpu_launches": 0})
    line["config"]["workload"] += " (host eager sample, extrapolated)"
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all", "fwdbwd", "fwd", "decode", "fx"],
                    default="all")
    ap.add_argument("--fx-layers", type=int, default=0,
                    help="override the layer count of the config-5 model (small runs)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--heads", type=int, default=0,
                    help="override the head count of configs 2-4 (small cases for profiling)")
    ap.add_argument("--decode-n-kv", type=int, default=0,
                    help="override config 4's cache length (small cases for profiling: the "
                         "visible rows per step, hence the traffic and grid, stay the same "
                         "while N_KV > S + W)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-weak", action="store_true",
                    help="skip the weak-scaling reference leg (N > 1)")
    ap.add_argument("--no-fx", action="store_true",
                    help="skip the config-5 FX end-to-end leg of the default run")
    args = ap.parse_args()
    if args.heads > 0:
        for cfg in (CFG2, CFG3, CFG4):
            cfg["H"] = args.heads
    if args.decode_n_kv > 0:
        CFG4["N"] = args.decode_n_kv
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    dist = Dist(args.gpus)
    dist.init()
    import sbfa_native as native
    native.lib()
    pk, src = peaks()
    line = base_line(args, dist.world)
    extra = {}
    if args.workload in ("all", "fwdbwd"):
        r = bench_fwdbwd(dist, args, pk, src)
        line.update({"value": round(r["value"], 3), "ms_per_step": round(r["ms"] / args.steps, 3),
                     "e2e": r["e2e"], "roofline": r["roofline"], "clocks": r["clocks"],
                     "gpu_launches": r["launches"]})
        line["config"]["timing"] = (r["timing"] + "; roofline and per-kernel times from an "
                                    "eager timed pass of the same step")
        start, stop, units = r["units"]
        extra["fwdbwd"] = {"kept_blocks": r["nnz"], "flops_fwd": r["flops_fwd"],
                           "units_rank0": [start, stop], "units_total": units,
                           "verify_rank0": r["verify"],
                           "per_kernel_ms": {k: round(v[0], 3) for k, v in r["per_kernel"].items()},
                           "per_kernel_ms_serialised_pass": {
                               k: round(v[0], 3) for k, v in r["per_kernel_iso"].items()},
                           "roofline_overlapped_pass": r["roofline_overlapped"],
                           "step_ms_rank0": [round(x, 3) for x in r["step_ms"]],
                           "host_enqueue_ms_rank0": [round(x, 3) for x in r["host_ms"]],
                           "timed_as": r["timing"],
                           "eager_pass": r["eager"]}
        _, mask = kept_blocks(CFG2)
        ex = executed_mma_flops(mask, CFG2, stop - start,
                                dq_gemms=1 if "dq_gemm_kernel" in r["per_kernel"] else 3)
        alg = {k: KERNEL_WORK[k] * r["flops_fwd"] * (stop - start) / units for k in ex}
        extra["fwdbwd"]["mma_flops_per_step_rank0"] = {
            k: {"executed": ex[k], "algorithmic": alg[k], "ratio": round(ex[k] / alg[k], 4)}
            for k in ex}
        if "weak" in r:
            extra["fwdbwd_weak_scaling"] = r["weak"]
    if args.workload in ("all", "fwd"):
        r = bench_fwd(dist, args, pk, src)
        extra["cfg3_prefill_fwd"] = {"value": round(r["value"], 3), "unit": "TFLOP/s",
                                     "ms_per_step": round(r["ms"], 3), "roofline": r["roofline"],
                                     "kept_blocks": r["nnz"], "gpu_launches": r["launches"],
                                     "clocks": r["clocks"], "units_rank0": list(r["units"][:2])}
        if args.workload == "fwd":
            line.update({"metric": "kept-block attn TFLOP/s fwd", "value": extra[
                "cfg3_prefill_fwd"]["value"], "roofline": r["roofline"], "dtype": "fp16"})
    if args.workload in ("all", "decode"):
        r = bench_decode(dist, args, pk, src)
        extra["cfg4_decode"] = {"value": round(r["value"], 2), "unit": "GB/s",
                                "ms_per_step": round(r["ms"], 4), "roofline": r["roofline"],
                                "kv_bytes_per_step": r["kv_bytes"], "n_kv": CFG4["N"],
                                "gpu_launches": r["launches"], "units_rank0": list(r["units"][:2])}
        extra["cfg4_decode_ring_cache"] = r["ring"]
        extra["cfg4_decode_gqa"] = r["gqa"]
        if args.workload == "decode":
            line.update({"metric": "decode KV GB/s", "unit": "GB/s", "value": extra[
                "cfg4_decode"]["value"], "roofline": r["roofline"], "dtype": "fp16"})
    if args.workload == "fx" or (args.workload == "all" and dist.world == 1 and not args.no_fx):
        r = bench_fx(dist, args, pk, src)
        extra["cfg5_fx_end_to_end"] = r
        if args.workload == "fx":
            line.update({"metric": "FX end-to-end tokens/s (fwd+bwd)", "unit": "tokens/s",
                         "value": r["tokens_per_s"], "ms_per_step": r["ms_per_step"],
                         "gpu_launches": r["gpu_launches"], "scaling": "weak", "config": {
                             "workload": r["config"], "global_batch": CFG5["B"] * dist.world,
                             "seq_len": CFG5["N"], "parallelism": f"replicas x{dist.world}"}})
    line["extra"] = extra
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline and \
            args.workload in ("all", "fwdbwd"):
        line["cpu_baseline"] = cpu_baseline_fwdbwd(budget_s=20.0)
    if dist.rank == 0:
        print(json.dumps(line))
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
