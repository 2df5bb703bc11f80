"""Benchmark of the BitSparse compression hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = compress one [8192, 14336] bf16 activation (relu of N(0,1), about
50% zeros; config 3) into a TensorBuffer arena with the fused kernel,
and reconstruct the tensor compressed in the previous step (two tensors
ping-pong, so the reconstruct reads data written ~470 MB of traffic earlier,
not L2-resident; every input is larger than the 126 MB L2).  ``value`` is
the algorithmic bytes of both operations over the device time of the K steps
(max over ranks); each rank runs its own batch (weak scaling, no collective
on the data path).

Also reported on the same line: ``e2e`` (the same step through the public
API with the dense input copied from pinned host memory and the
reconstruction copied back inside the timed region; the copies run on their
own streams, so one step's upload overlaps the previous step's download),
``roofline`` of the
dominant kernel (compress), ``cpu_baseline`` (the CPU oracle on the host
cores), the sparsity / structure ``sweep`` of config 3, and ``mlp``: sparse
FFN fwd+bwd tokens/s (configs 2 and 4) beside a dense-activation torch FFN.

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle port; the reference itself is Python + Triton and runs on a CPU only
through the Triton interpreter, which is not installed on the GPU box) on
the same workload and prints the same line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M_C3, N_C3 = 8192, 14336
METRIC = "compress/reconstruct GB/s (% HBM peak); sparse-MLP fwd+bwd tokens/s"
WORKLOAD = ("config3 compress+reconstruct round trip, [8192,14336] bf16 relu(N(0,1)) "
            "~50% sparse, TensorBuffer arena, 64x64 tiles")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def ncu_traffic(kernel: str):
    """DRAM bytes per launch from a committed ncu summary, or None."""
    f = ROOT / "profiles" / "traffic.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region: a thread
    runs one-shot queries back to back (about every 100 ms)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines = []
        self._stop = threading.Event()

    def _query(self):
        try:
            out = subprocess.run(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits"],
                capture_output=True, text=True, timeout=5).stdout
            self.lines.extend(l.strip() for l in out.splitlines() if l.strip())
        except (OSError, subprocess.SubprocessError):
            pass

    def _run(self):
        while not self._stop.is_set():
            self._query()
            self._stop.wait(0.1)

    def __enter__(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self.t.join(10)
        if not self.lines:  # a very short timed region: take one sample anyway
            self._query()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------
def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(rows: int, steps: int, warmup: int):
    from oracle.cpu_baseline import CpuRoundTrip

    c = CpuRoundTrip(rows, N_C3)
    try:
        gbs, dt = c.measure(steps, warmup)
    finally:
        c.close()
    return gbs, dt, c.workers


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    rows = 2048  # bounded sample of the [8192, 14336] workload (1/4 of its rows)
    gbs, dt, cores = cpu_baseline(rows, args.steps, args.warmup)
    sample = (f"oracle round trip (the NumPy port of the reference's algorithm, not the "
              f"reference's Triton code, which runs on a CPU only in the Triton "
              f"interpreter) of a [{rows},{N_C3}] bf16 slice (1/4 of the config-3 rows; "
              f"the unit is GB/s, so a slice is a fair sample) per step, {cores} worker "
              f"processes on {os.cpu_count()} host threads, CPU {cpu_model()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_rows": rows},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def make_relu_bf16(M, N, mu, seed, device, variant="A", target=0.5):
    """relu of a seeded N(mu, 1) bf16 [M, N] tensor; ``target`` is the
    SPARSITY (fraction of zeros) the variant aims at.

    A: the mean mu sets the sparsity (mu = -ndtri(target)).
    B: each row's density is drawn from Beta(2,2) scaled around 1 - target.
    C: a fraction target / 2 of the 64-column strips is zeroed outright and
       the rest is N(mu', 1) with mu' chosen so that the total sparsity is
       target (half of the zeros come from whole strips)."""
    import torch

    import numpy as np

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, N, generator=g, device=device, dtype=torch.float32)
    if variant == "B":  # per-row density ~ Beta(2,2) scaled around the target
        d = torch.from_numpy(np.random.default_rng(seed).beta(2.0, 2.0, (M, 1))).float()
        d = d.to(device)
        dens = (2 * (1 - target) * d).clamp(1e-4, 0.9999)
        mu_row = torch.special.ndtri(dens)  # P(N(mu,1) > 0) = dens
        x = x + mu_row
    elif variant == "C":
        zf = target / 2
        rest = (target - zf) / (1 - zf)  # sparsity of the strips left alone
        x = x - float(torch.special.ndtri(torch.tensor(rest, dtype=torch.float64)))
        strips = torch.rand(N // 64, generator=g, device=device) < zf
        x.view(M, N // 64, 64)[:, strips, :] = -1.0
    else:
        x = x + mu
    return x.relu_().to(torch.bfloat16)


def compress_bytes(M, N, nnz, elt=2):
    T = ((M + 63) // 64) * ((N + 63) // 64)
    return M * N * elt + M * N // 8 + nnz * elt + 4 * (T + 1)


def time_round_trips(xs, bufs, outs, steps, sps=None):
    """Run `steps` ping-pong steps: step i compresses xs[i % 2] and
    reconstructs the tensor compressed by the step before (``sps`` carries
    it across calls).  Returns (sps, [(e0, e1, e2, reconstructed?)])."""
    import torch
    from bitsparse_b200.src.functions import dense_to_tilesparse
    from bitsparse_b200.src.operators import unpack_batch_

    st = torch.cuda.current_stream()
    sps = sps if sps is not None else [None, None]
    ev = []
    for i in range(steps):
        a = i & 1
        bufs[a].offset.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        sps[a] = dense_to_tilesparse(xs[a], None, bufs[a])
        e1.record(st)
        prev = sps[1 - a]
        if prev is not None:
            unpack_batch_(prev, outs[1 - a], 0, prev.grid_n, prev.shape[1], prev.shape[0],
                          prev.grid_m * prev.grid_n)
        e2.record(st)
        ev.append((e0, e1, e2, prev is not None))
    return sps, ev


class _DenseReluLinearFP8:
    """The FP8 ReLU / ReLU^2 FFN half of the reference (lib_sparse/layers.py:
    20-66, 100-151) with the activation kept DENSE: the same FP8 GEMM calls
    (``bitsparse_b200.fp8.matmul``), the saved activation ``to_fp8(h)`` as a
    dense e4m3 tensor.  The config-4 baseline that differs from the
    compressed FFN only in how the activation is stored."""

    @staticmethod
    def make():
        import torch
        from bitsparse_b200.fp8 import matmul, to_fp8

        class F(torch.autograd.Function):
            @staticmethod
            def forward(ctx, z, W, relu2):
                ctx.relu2 = relu2
                ctx.save_for_backward(W)
                h = z.relu_()
                h_st, scale = to_fp8(h)
                ctx.h_st, ctx.scale = h_st, scale
                if relu2:
                    return matmul(h.square_(), W.T, True)
                return matmul(h_st, W.T, True, a_scale=scale)

            @staticmethod
            def backward(ctx, go):
                W = ctx.saved_tensors[0]
                h, scale = ctx.h_st, ctx.scale
                go8, gscale = to_fp8(go.contiguous())
                r = h.float() * scale
                if ctx.relu2:
                    gW = matmul(go8.T, (r * r).to(torch.bfloat16), True, a_scale=gscale)
                    gh = matmul(go8, W, True, a_scale=gscale)
                    gz = (gh.float() * (2.0 * r)).to(torch.bfloat16)
                else:
                    gW = matmul(go8.T, h, True, a_scale=gscale, b_scale=scale)
                    gz = matmul(go8, W, True, a_scale=gscale) * (r > 0)
                return gz, gW, None

        return F


def mlp_bench(cfg, steps, warmup, device):
    """Sparse FFN fwd+bwd tokens/s vs a dense-activation torch FFN."""
    import torch
    from bitsparse_b200.layers import FFNRelu, FFNRelu2

    T, d, H, relu2, storage = cfg["tokens"], cfg["d"], cfg["H"], cfg["relu2"], cfg["storage"]
    g = torch.Generator(device=device).manual_seed(123)
    x = torch.randn(T, d, generator=g, device=device).to(torch.bfloat16)
    W1 = (0.02 * torch.randn(H, d, generator=g, device=device)).to(torch.bfloat16)
    W2 = (0.02 * torch.randn(d, H, generator=g, device=device)).to(torch.bfloat16)
    b2 = torch.zeros(d, device=device, dtype=torch.bfloat16)
    with torch.no_grad():
        z = (x @ W1.T).float()
        b1 = (-cfg["bias_sigma"] * z.std()).to(torch.bfloat16).expand(H).contiguous()
    gy = torch.randn(T, d, generator=g, device=device).to(torch.bfloat16)
    params = [t.requires_grad_() for t in (x, W1, W2, b1, b2)]

    from bitsparse_b200 import TensorBuffer

    elt = 1 if storage != torch.bfloat16 else 2
    arena = TensorBuffer(T * H * elt, device=device, dtype=storage)

    def sparse_step(buf=None):
        kw = {"storage_dtype": storage} if relu2 else {"dtype": storage}
        if buf is not None:
            buf.offset.zero_()  # one activation per step: reuse the arena
            kw["sparse_data"] = buf
        y = (FFNRelu2 if relu2 else FFNRelu).apply(*params, **kw)
        y.backward(gy)

    def dense_step():
        h = torch.relu(params[0] @ params[1].T + params[3])
        if relu2:
            h = h * h
        y = h @ params[2].T + params[4]
        y.backward(gy)

    fp8 = storage != torch.bfloat16
    if fp8:
        from bitsparse_b200.fp8 import matmul as mm8
        DenseFP8 = _DenseReluLinearFP8.make()

    def dense_fp8_step():
        z = mm8(params[0], params[1].T, True) + params[3]
        y = DenseFP8.apply(z, params[2], relu2) + params[4]
        y.backward(gy)

    def graphed(fn):
        """fn captured once in a CUDA graph (launch overhead removed)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g.replay

    out = {}
    arms = [("sparse", sparse_step), ("sparse_arena", lambda: sparse_step(arena)),
            ("dense", dense_step),
            ("sparse_arena_graph", graphed(lambda: sparse_step(arena))),
            ("dense_graph", graphed(dense_step))]
    if fp8:
        arms.append(("dense_fp8", dense_fp8_step))
    for name, fn in arms:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        out[name] = {"tokens_per_s": T / ms * 1e3, "ms_per_step": ms,
                     "peak_extra_mem_mb": (torch.cuda.max_memory_allocated() - base) / 2**20}
    with torch.no_grad():
        sparsity = (torch.relu(x @ W1.T + b1) == 0).float().mean().item()
    out["sparsity"] = sparsity
    out["speedup_vs_dense"] = out["sparse"]["tokens_per_s"] / out["dense"]["tokens_per_s"]
    out["speedup_arena_vs_dense"] = (out["sparse_arena"]["tokens_per_s"]
                                     / out["dense"]["tokens_per_s"])
    out["speedup_graph_vs_dense_graph"] = (out["sparse_arena_graph"]["tokens_per_s"]
                                           / out["dense_graph"]["tokens_per_s"])
    if fp8:  # like for like: the same FP8 GEMMs, only the activation storage differs
        out["speedup_vs_dense_fp8"] = (out["sparse"]["tokens_per_s"]
                                       / out["dense_fp8"]["tokens_per_s"])
        out["speedup_arena_vs_dense_fp8"] = (out["sparse_arena"]["tokens_per_s"]
                                             / out["dense_fp8"]["tokens_per_s"])
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    import bitsparse_b200 as B
    from bitsparse_b200 import TensorBuffer, _lib
    from bitsparse_b200.src.functions import dense_to_tilesparse
    from bitsparse_b200.src.operators import unpack_batch_

    _lib.load()
    M, N = M_C3, N_C3
    xs = [make_relu_bf16(M, N, 0.0, 1000 * rank + i, dev) for i in range(2)]
    bufs = [TensorBuffer(M * N * 2, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    outs = [torch.empty_like(x) for x in xs]

    # warm-up (an even count, so the timed steps start with xs[0] and have a
    # predecessor to reconstruct), then more warm-up rounds of 10 steps until
    # the compress launch time has settled (the median of a round within 2%
    # of the previous round's), at most 20 rounds
    sps, _ = time_round_trips(xs, bufs, outs, max(args.warmup, 3) // 2 * 2 + 2)
    torch.cuda.synchronize()
    prev = None
    for _ in range(20):
        sps, ev = time_round_trips(xs, bufs, outs, 10, sps)
        torch.cuda.synchronize()
        med = statistics.median(e0.elapsed_time(e1) for e0, e1, _, _ in ev)
        if prev is not None and abs(med - prev) <= 0.02 * prev:
            break
        prev = med
    nnz = [int((x > 0).sum().item()) for x in xs]
    # step i compresses xs[i % 2] and reconstructs xs[(i - 1) % 2]
    step_bytes = [compress_bytes(M, N, nnz[i & 1]) + compress_bytes(M, N, nnz[1 - (i & 1)])
                  for i in range(args.steps)]

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record()
        sps, ev = time_round_trips(xs, bufs, outs, args.steps, sps)
        t1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = t0.elapsed_time(t1)
    comp_ms = [e0.elapsed_time(e1) for e0, e1, _, _ in ev]
    unp_ms = [e1.elapsed_time(e2) for _, e1, e2, has in ev if has]
    bytes_total = sum(step_bytes)
    ms_t = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = ms_t.item()
    value = bytes_total * world / (ms_max * 1e-3) / 1e9

    # correctness of the last reconstructs (outside the timed region)
    for a in range(2):
        if not torch.equal(outs[a], xs[a]):
            raise RuntimeError("round trip mismatch")
    B.check_status(dev)

    hbm, bf16_peak, peak_kind = peaks()
    comp_avg = statistics.mean(comp_ms)
    comp_alg = compress_bytes(M, N, statistics.mean(nnz))
    achieved = comp_alg / (comp_avg * 1e-3) / 1e9
    unp_avg = statistics.mean(unp_ms)
    traffic = ncu_traffic("onepass_kernel")

    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "shape": [M, N], "sparsity": 1 - nnz[0] / (M * N),
                   "l2": "inputs larger than L2 (235 MB each, 2 ping-pong tensors)",
                   "parallelism": f"dp{world} (row-independent batches, no collective)"},
        "pct_hbm_peak": value / world / hbm,
        "roofline": {"bound": "hbm", "kernel": "compress (bs_compress fused)",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": f"{peak_kind} (burst copy)",
                     "traffic": traffic,
                     "alg_bytes_per_launch": comp_alg, "avg_launch_ms": comp_avg,
                     "median_launch_ms": statistics.median(comp_ms),
                     "frac_at_median": comp_alg / (statistics.median(comp_ms) * 1e-3) / 1e9 / hbm},
        "reconstruct": {"achieved": comp_alg / (unp_avg * 1e-3) / 1e9, "avg_launch_ms": unp_avg,
                        "median_launch_ms": statistics.median(unp_ms),
                        "frac": comp_alg / (unp_avg * 1e-3) / 1e9 / hbm},
        "clocks": clk.summary(),
        "gpu_launches": 2 * args.steps,
    }

    # ---- e2e: host buffers through the public API --------------------------
    hx = [x.cpu().pin_memory() for x in xs]
    hout = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dx = [torch.empty_like(x) for x in xs]

    # A streaming pipeline over double buffers: step i's host->device copy
    # (stream s_in), its compress + reconstruct (s_run) and its
    # device->host copy (s_out) are ordered by events, so step i+1's input
    # copy overlaps step i's output copy (PCIe is full duplex).  Every step
    # still moves its own input in and its own result out.
    s_in, s_run, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_run = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]  # dx[a] read by its last run
    used = [False, False]

    def e2e_step(i):
        a = i & 1
        with torch.cuda.stream(s_in):
            if used[a]:
                s_in.wait_event(ev_free[a])
            dx[a].copy_(hx[a], non_blocking=True)
            ev_in[a].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(ev_in[a])
            if used[a]:
                s_run.wait_event(ev_out[a])  # outs[a] copied out by its last step
            bufs[a].offset.zero_()
            sp = dense_to_tilesparse(dx[a], None, bufs[a])
            ev_free[a].record(s_run)
            unpack_batch_(sp, outs[a], 0, sp.grid_n, N, M, sp.grid_m * sp.grid_n)
            ev_run[a].record(s_run)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_run[a])
            hout[a].copy_(outs[a], non_blocking=True)
            ev_out[a].record(s_out)
        used[a] = True

    def drain():
        cur = torch.cuda.current_stream(dev)
        for st in (s_in, s_run, s_out):
            cur.wait_stream(st)

    for i in range(2):
        e2e_step(i)
    drain()
    torch.cuda.synchronize()
    ksteps = max(2, args.steps // 2)
    if world > 1:
        dist.barrier()
    t0.record()
    for st in (s_in, s_run, s_out):
        st.wait_stream(torch.cuda.current_stream(dev))
    for i in range(ksteps):
        e2e_step(i)
    drain()
    t1.record()
    torch.cuda.synchronize()
    # the pipeline returned every step's round trip to the host
    assert torch.equal(hout[(ksteps - 1) & 1], hx[(ksteps - 1) & 1])
    e_ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e_bytes = sum(2 * compress_bytes(M, N, nnz[i & 1]) for i in range(ksteps))
    line["e2e"] = {"value": e_bytes * world / (e_ms.item() * 1e-3) / 1e9, "unit": "GB/s",
                   "h2d_bytes_per_step": M * N * 2, "d2h_bytes_per_step": M * N * 2,
                   "ms_per_step": e_ms.item() / ksteps}

    del hx, hout, dx
    torch.cuda.empty_cache()

    # ---- multi-GPU sections (every rank) -----------------------------------
    if not args.no_extras and not args.sweep_only and not args.no_train:
        del xs, bufs, outs, sps
        torch.cuda.empty_cache()
        line["train"] = train_suite(dev, world, rank)
        xs = [make_relu_bf16(M, N, 0.0, 1000 * rank + i, dev) for i in range(2)]
        bufs = [TensorBuffer(M * N * 2, device=dev, dtype=torch.bfloat16) for _ in range(2)]
        outs = [torch.empty_like(x) for x in xs]

    # ---- extras on rank 0 at N = 1: sweep, MLP, CPU baseline ----------------
    # (per-GPU measurements; at N > 1 the other ranks would only wait)
    if rank == 0 and world == 1 and not args.no_extras:
        sweep = {}
        for variant in ("A", "B", "C"):
            for target, mu in ((0.5, 0.0), (0.7, -0.5244), (0.9, -1.2816), (0.95, -1.6449),
                               (0.99, -2.3263)):
                if variant != "A" and target not in (0.5, 0.9):
                    continue
                x2 = [make_relu_bf16(M, N, mu, 7 + i, dev, variant, target)
                      for i in range(2)]
                s2, _ = time_round_trips(x2, bufs, outs, 4)
                torch.cuda.synchronize()
                nz = [int((x > 0).sum().item()) for x in x2]
                _, ev2 = time_round_trips(x2, bufs, outs, 10, s2)
                torch.cuda.synchronize()
                c = statistics.mean(e0.elapsed_time(e1) for e0, e1, _, _ in ev2)
                u = statistics.mean(e1.elapsed_time(e2) for _, e1, e2, h in ev2 if h)
                by = compress_bytes(M, N, statistics.mean(nz))
                sweep[f"{variant}{int(target * 100)}"] = {
                    "sparsity": 1 - statistics.mean(nz) / (M * N),
                    "compress_GBs": by / c / 1e6, "reconstruct_GBs": by / u / 1e6,
                    "compress_frac": by / c / 1e6 / hbm, "reconstruct_frac": by / u / 1e6 / hbm}
                del x2
        line["sweep"] = sweep
        del xs, bufs, outs
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_extras and not args.sweep_only:
        line["mlp"] = mlp_suite(dev)
        if world == 1:
            gbs, dt, cores = cpu_baseline(2048, 1, 1)
            line["cpu_baseline"] = {
                "value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"oracle round trip (NumPy port of the reference's algorithm) of a "
                          f"[2048,{N_C3}] bf16 slice, {dt:.2f} s/step, {cores} worker "
                          f"processes, CPU {cpu_model()}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _max_over_ranks(v: float, world: int, dev) -> float:
    import torch
    import torch.distributed as dist
    if world == 1:
        return v
    t = torch.tensor([v], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def dp_train(dev, world, rank, compressed, steps=4, warmup=2, arena_fraction=0.0):
    """Config 5: one data-parallel training step (forward, backward with the
    gradients summed over the ranks by NCCL all-reduce overlapped with the
    backward pass, AdamW) of the 24-layer d1024 decoder on a global batch of
    64 x 1024 synthetic tokens (64 / world sequences per rank: strong
    scaling).  Returns tokens/s (device time, max over ranks) and the peak
    memory the forward pass adds on top of parameters, gradients and
    optimizer state (the saved activations, logits included)."""
    import torch
    import torch.distributed as dist
    from bitsparse_b200.decoder import Decoder, DecoderConfig
    from bitsparse_b200.distributed import GradAllReduce

    cfg = DecoderConfig(compressed=compressed, arena_fraction=arena_fraction)
    torch.manual_seed(0)  # the same initial weights on every rank
    model = Decoder(cfg).to(device=dev, dtype=torch.bfloat16)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-5, fused=True)
    red = GradAllReduce(model.parameters()) if world > 1 else None
    B = max(1, 64 // world)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    tok = torch.randint(0, cfg.vocab, (B, cfg.seq + 1), generator=g, device=dev)
    x, y = tok[:, :-1], tok[:, 1:]

    def step():
        loss = model(x, y)
        loss.backward()
        if red is not None:
            red.wait()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    loss = model(x, y)
    torch.cuda.synchronize()
    fwd_peak = torch.cuda.max_memory_allocated(dev) - base
    loss.backward()
    if red is not None:
        red.wait()
    opt.step()
    opt.zero_grad(set_to_none=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        last = step()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
    arena_mb = 0.0
    if model.arena is not None:  # preallocated, so outside fwd_peak: count it here
        import bitsparse_b200 as B_
        B_.check_status(dev)  # no capacity overflow
        arena_mb = model.arena.vals.numel() * model.arena.vals.element_size() / 2**20
    out = {"tokens_per_s": B * world * cfg.seq / ms * 1e3, "ms_per_step": ms,
           "local_batch": B, "peak_forward_mem_mb": fwd_peak / 2**20 + arena_mb,
           "arena_mb": arena_mb,
           "loss_per_token": float(last.item()) / (B * cfg.seq)}
    if red is not None:
        red.remove()
    del model, opt, red
    torch.cuda.empty_cache()
    return out


def c4_sharded(dev, world, rank, steps=5, warmup=2, bias_sigma=0.0):
    """Config 4 token-sharded: the 16384 tokens split over the ranks, each
    rank runs the compressed ReLU^2 FFN (e4m3 storage) forward and backward
    on its tokens and the weight / bias gradients are summed over the ranks
    (GradAllReduce, overlapped with the backward pass)."""
    import torch
    import torch.distributed as dist
    from bitsparse_b200.distributed import GradAllReduce
    from bitsparse_b200.layers import FFNRelu2

    d, H = 4096, 16384
    T = 16384 // world
    gw = torch.Generator(device=dev).manual_seed(123)  # shared weights
    W1 = (0.02 * torch.randn(H, d, generator=gw, device=dev)).to(torch.bfloat16)
    W2 = (0.02 * torch.randn(d, H, generator=gw, device=dev)).to(torch.bfloat16)
    gx = torch.Generator(device=dev).manual_seed(500 + rank)
    x = torch.randn(T, d, generator=gx, device=dev).to(torch.bfloat16)
    gy = torch.randn(T, d, generator=gx, device=dev).to(torch.bfloat16)
    with torch.no_grad():
        z = (x @ W1.T).float()
        b1 = (-bias_sigma * z.std()).to(torch.bfloat16).expand(H).contiguous()
        del z
    b2 = torch.zeros(d, device=dev, dtype=torch.bfloat16)
    params = [t.requires_grad_() for t in (x, W1, W2, b1, b2)]
    red = GradAllReduce(params[1:]) if world > 1 else None

    def step():
        y = FFNRelu2.apply(*params, storage_dtype=torch.float8_e4m3fn)
        y.backward(gy)
        if red is not None:
            red.wait()
        for p in params:
            p.grad = None

    for _ in range(warmup):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
    out = {"tokens_per_s": 16384 / ms * 1e3, "ms_per_step": ms, "tokens_per_rank": T}
    if red is not None:
        red.remove()
    return out


def train_suite(dev, world, rank):
    """Multi-GPU sections, run by every rank: config 5 (DP decoder step,
    compressed vs dense MLP activations) and config 4 token-sharded."""
    out = {"scaling": "strong (global batch fixed)", "world": world}
    out["config5_dp_decoder_compressed"] = dp_train(dev, world, rank, True)
    # the same with one TensorBuffer arena for every layer's values (sized
    # for 60% density: random-init ReLU activations are about 50% dense)
    out["config5_dp_decoder_compressed_arena"] = dp_train(dev, world, rank, True,
                                                          arena_fraction=0.6)
    out["config5_dp_decoder_dense"] = dp_train(dev, world, rank, False)
    dn = out["config5_dp_decoder_dense"]
    for k in ("", "_arena"):
        c = out["config5_dp_decoder_compressed" + k]
        out["config5_speedup_vs_dense" + k] = c["tokens_per_s"] / dn["tokens_per_s"]
        out["config5_activation_mem_ratio" + k] = (c["peak_forward_mem_mb"]
                                                   / dn["peak_forward_mem_mb"])
    out["config4_token_sharded_relu2_fp8"] = c4_sharded(dev, world, rank)
    return out


def mlp_suite(dev):
    import torch

    return {
            "config2_gpt2_small_relu_bf16": mlp_bench(
                {"tokens": 8 * 1024, "d": 768, "H": 3072, "relu2": False,
                 "storage": torch.bfloat16, "bias_sigma": 1.0}, 50, 10, dev),
            "config2_relu_bf16_90pct_sparse": mlp_bench(
                {"tokens": 8 * 1024, "d": 768, "H": 3072, "relu2": False,
                 "storage": torch.bfloat16, "bias_sigma": 1.2816}, 50, 10, dev),
            # the nanoGPT MLP's own activation (ReLU^2), bf16 storage
            "config2_gpt2_small_relu2_bf16": mlp_bench(
                {"tokens": 8 * 1024, "d": 768, "H": 3072, "relu2": True,
                 "storage": torch.bfloat16, "bias_sigma": 1.0}, 50, 10, dev),
            "config4_nemotron_relu2_fp8": mlp_bench(
                {"tokens": 16384, "d": 4096, "H": 16384, "relu2": True,
                 "storage": torch.float8_e4m3fn, "bias_sigma": 0.0}, 5, 2, dev),
            "config4_nemotron_relu2_fp8_90pct_sparse": mlp_bench(
                {"tokens": 16384, "d": 4096, "H": 16384, "relu2": True,
                 "storage": torch.float8_e4m3fn, "bias_sigma": 1.2816}, 5, 2, dev),
    }


def gemm_case():
    """Small case for ncu captures of K3 (the tcgen05 GEMM with the ReLU mask
    in its epilogue): the config-2 backward shape (grad_z = grad_y @ W2
    masked by h, [8192 x 768] @ [768 x 3072]) and a square 8192^3 product,
    each with and without the mask, checked against torch."""
    import torch
    from bitsparse_b200.src.functions import dense_to_tilesparse
    from bitsparse_b200.src.operators import mask_with_bitmask_, matmul_relu_mask

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    for M, N, K in ((8192, 3072, 768), (8192, 8192, 8192)):
        a = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn(K, N, generator=g, device=dev).to(torch.bfloat16)
        h = torch.randn(M, N, generator=g, device=dev).relu().to(torch.bfloat16)
        sp = dense_to_tilesparse(h, None)
        for _ in range(2):
            out = matmul_relu_mask(a, b, sp)
            plain = matmul_relu_mask(a, b)
        ref = mask_with_bitmask_((a.float() @ b.float()).to(torch.bfloat16), sp).float()
        err = (out.float() - ref).abs().max().item()
        if err > 1e-2 * ref.abs().max().item() or not bool(torch.all(out[h == 0] == 0)):
            raise RuntimeError(f"gemm case mismatch at {(M, N, K)}: {err}")
        del plain
    import bitsparse_b200 as B
    B.check_status(dev)
    print("gemm case ok")


def kernel_cases(which: str):
    """Small ncu capture cases of the kernels added beside K1 / K2 / K3:
    "fp8" -- the tcgen05 FP8 GEMM at 8192^3 (e4m3, tensor-wise scales);
    "relu2" -- the bf16 GEMM with the ReLU^2 gradient in its epilogue at the
    config-2 backward shape (8192 x 768 @ 768 x 3072, h 84% sparse);
    "sparse_recon" -- the persistent reconstruct of an [8192, 8192] bf16
    tensor at 99% sparsity (the sparse-chunk scatter path); "dw" -- the
    fused reconstruct + tcgen05 weight-gradient GEMM at the config-2
    backward shape (go^T [768 x 8192] @ h [8192 x 3072], h 50% sparse),
    checked against the fp32 product and timed against unpack + cuBLAS; "fp8_compress" -- the one-pass FP8
    quantise + compress of an [8192, 8192] bf16 tensor, plain and with bias,
    ReLU and the square side output.  Each runs its kernel twice and checks
    the result."""
    import torch
    from bitsparse_b200 import TensorBuffer
    from bitsparse_b200.src.functions import dense_to_tilesparse
    from bitsparse_b200.src.operators import (matmul_relu2_grad, matmul_relu_mask,
                                              relu2_grad_sparse_, unpack_batch_)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if which == "fp8":
        from bitsparse_b200.fp8 import gemm_fp8
        n = 8192
        a = torch.randn(n, n, generator=g, device=dev).to(torch.float8_e4m3fn)
        bt = torch.randn(n, n, generator=g, device=dev).to(torch.float8_e4m3fn)
        s1 = torch.tensor(1.0, device=dev)
        for _ in range(2):
            out = gemm_fp8(a, bt, s1, s1)
        ref = a[:256].float() @ bt.float().T
        if (out[:256].float() - ref).abs().max() > 1e-2 * ref.abs().max():
            raise RuntimeError("fp8 gemm case mismatch")
        import torch.nn.functional as F

        def ev(fn, k=20):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(k):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / k * 1e3

        ours = ev(lambda: gemm_fp8(a, bt, s1, s1))
        cub = ev(lambda: F.scaled_mm(a, bt.T, scale_a=s1, scale_b=s1, output_dtype=torch.bfloat16,
                                     scale_recipe_a=F.ScalingType.TensorWise,
                                     scale_recipe_b=F.ScalingType.TensorWise))
        fl = 2.0 * n ** 3
        print(f"fp8 {n}^3: tcgen05 {ours:.1f} us ({fl / ours / 1e6:.0f} TFLOP/s), "
              f"cuBLASLt scaled_mm {cub:.1f} us ({fl / cub / 1e6:.0f} TFLOP/s)")
    elif which == "relu2":
        M, N, K = 8192, 3072, 768
        a = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn(K, N, generator=g, device=dev).to(torch.bfloat16)
        h = (torch.randn(M, N, generator=g, device=dev) - 1.0).relu().to(torch.bfloat16)
        sp = dense_to_tilesparse(h, None)
        for _ in range(2):
            out = matmul_relu2_grad(a, b, sp)
        if not torch.equal(out, relu2_grad_sparse_(matmul_relu_mask(a, b), sp)):
            raise RuntimeError("relu2 gemm case mismatch")
        import os
        if os.environ.get("BS_CASE_TIMING", "1") == "1":
            def ev(fn, k=50):
                for _ in range(5):
                    fn()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(k):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) / k * 1e3
            fused = ev(lambda: matmul_relu2_grad(a, b, sp))
            two = ev(lambda: relu2_grad_sparse_(matmul_relu_mask(a, b), sp))
            cub = ev(lambda: relu2_grad_sparse_(a @ b, sp))
            print(f"ReLU^2 dX {M}x{K} @ {K}x{N}: fused epilogue {fused:.1f} us, tcgen05 GEMM + "
                  f"relu2_grad {two:.1f} us, cuBLAS + relu2_grad {cub:.1f} us")
    elif which == "dw":
        import os
        import bitsparse_b200.src.sparse_matmul as SM
        from bitsparse_b200.src.operators import matmul_unpack_dw
        T, D, H = 8192, 768, 3072
        go = torch.randn(T, D, generator=g, device=dev).to(torch.bfloat16)
        h = torch.randn(T, H, generator=g, device=dev).relu().to(torch.bfloat16)
        sp = dense_to_tilesparse(h, None)
        for _ in range(2):
            out = matmul_unpack_dw(go.T, sp)
        ref = go.float().T @ h.float()  # (K is split here: partial sums in another order)
        if (out.float() - ref).abs().max() > 1e-2 * ref.abs().max():
            raise RuntimeError("fused dW case mismatch")
        if os.environ.get("BS_CASE_TIMING", "1") == "1":
            def ev(fn, k=20):
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(k):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) / k * 1e3
            SM.FUSED_DW = False
            for (T2, D2, H2) in ((T, D, H), (8192, 1024, 4096), (16384, 4096, 16384)):
                if (T2, D2, H2) != (T, D, H):
                    go = torch.randn(T2, D2, generator=g, device=dev).to(torch.bfloat16)
                    h = torch.randn(T2, H2, generator=g, device=dev).relu().to(torch.bfloat16)
                    sp = dense_to_tilesparse(h, None)
                fused = ev(lambda: matmul_unpack_dw(go.T, sp))
                unf = ev(lambda: SM.AspB(go.T, sp))
                cub = ev(lambda: go.T @ h)
                print(f"dW {D2}x{T2}x{H2}: fused {fused:.1f} us, unpack + cuBLAS {unf:.1f} us, "
                      f"cuBLAS alone {cub:.1f} us")
    elif which == "tile_scaled":
        # per-tile FP8 scale mode: one pass (tile amax, quantise, compress)
        # against the per-tensor path (amax pass + quantise + compress), and
        # the dequantising reconstruct; fraction of the measured HBM peak
        from bitsparse_b200.src.functions import relu_to_tilesparse_fp8
        from bitsparse_b200.src.operators import compress_fp8_tile_scaled, unpack_tile_scaled_
        n = 8192
        x = torch.randn(n, n, generator=g, device=dev).relu().to(torch.bfloat16)
        buf = TensorBuffer(n * n, device=dev, dtype=torch.float8_e4m3fn)

        def ts():
            buf.offset.zero_()
            return compress_fp8_tile_scaled(x, buf)
        sp = ts()
        out = torch.empty(n, n, device=dev, dtype=torch.bfloat16)
        unpack_tile_scaled_(sp, out)
        # half an e4m3 step (2^-4 relative in the normal range, 2^-10 of the
        # tile's scale in the subnormal range) plus the output's bf16 rounding
        sfull = sp.tile_scales.view(sp.grid_m, sp.grid_n).repeat_interleave(64, 0) \
            .repeat_interleave(64, 1)[:n, :n]
        tol = x.float().abs() * (2.0 ** -4 + 2.0 ** -8) + sfull * 2.0 ** -10 * 1.01
        if bool(((out.float() - x.float()).abs() > tol).any()):
            raise RuntimeError("tile-scaled round trip error")

        def ev(fn, k=20):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(k):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / k * 1e3
        peak = peaks()[0]
        nnz = int(sp.prefix[-1].item())
        T = sp.grid_m * sp.grid_n
        c_bytes = n * n * 2 + n * n / 8 + nnz + 4 * (T + 1) + 4 * T
        r_bytes = n * n / 8 + nnz + 4 * (T + 1) + 4 * T + n * n * 2
        t_ts = ev(ts)

        def pt():
            buf.offset.zero_()
            relu_to_tilesparse_fp8(x, sparse_data=buf)
        t_pt = ev(pt)
        t_un = ev(lambda: unpack_tile_scaled_(sp, out))
        print(f"tile-scaled compress {t_ts:.1f} us = {c_bytes / t_ts / 1e3:.0f} GB/s "
              f"({c_bytes / t_ts / 1e3 / peak:.2f} of peak); per-tensor to_fp8 + compress "
              f"{t_pt:.1f} us; dequantising reconstruct {t_un:.1f} us = "
              f"{r_bytes / t_un / 1e3:.0f} GB/s ({r_bytes / t_un / 1e3 / peak:.2f})")
    elif which == "fp8_compress":
        from bitsparse_b200.fp8 import to_fp8
        from bitsparse_b200.src.functions import relu_to_tilesparse_fp8
        from bitsparse_b200.src.operators import compress_bias_relu_fp8
        n = 8192
        x = torch.randn(n, n, generator=g, device=dev).to(torch.bfloat16)
        b = (0.1 * torch.randn(n, generator=g, device=dev)).to(torch.bfloat16)
        h = torch.relu(x + b)
        buf = TensorBuffer(n * n, device=dev, dtype=torch.float8_e4m3fn)
        for _ in range(2):
            buf.offset.zero_()
            side, ss, sp = compress_bias_relu_fp8(x, b, buf, False, square=True)
            buf.offset.zero_()
            q, sp2 = relu_to_tilesparse_fp8(h, sparse_data=buf)
        if not torch.equal(side.view(torch.uint8), to_fp8(h * h)[0].view(torch.uint8)) or \
                not torch.equal(q.view(torch.uint8), to_fp8(h)[0].view(torch.uint8)):
            raise RuntimeError("fp8 compress case mismatch")
        from bitsparse_b200.fp8 import estimate_exact
        print("quantiser estimate path (h, h*h, relu case):", estimate_exact(sp.scale.reshape(())),
              estimate_exact(ss.reshape(())), estimate_exact(sp2.scale.reshape(())))
    else:
        M = N = 8192
        x = make_relu_bf16(M, N, -2.3263, 0, dev)
        buf = TensorBuffer(M * N * 2, device=dev, dtype=torch.bfloat16)
        sp = dense_to_tilesparse(x, None, buf)
        out = torch.empty_like(x)
        for _ in range(2):
            unpack_batch_(sp, out, 0, sp.grid_n, N, M, sp.grid_m * sp.grid_n)
        if not torch.equal(out, x):
            raise RuntimeError("sparse reconstruct case mismatch")
    torch.cuda.synchronize()
    print(which, "case ok")


def profile_case():
    """Small case for ncu captures: compress + reconstruct of one [8192, 8192]
    bf16 relu(N(0,1)) tensor (134 MB, above L2) into a TensorBuffer, 3 times."""
    import torch
    from bitsparse_b200 import TensorBuffer
    from bitsparse_b200.src.functions import dense_to_tilesparse
    from bitsparse_b200.src.operators import unpack_batch_

    M = N = 8192
    x = make_relu_bf16(M, N, 0.0, 0, torch.device("cuda", 0))
    buf = TensorBuffer(M * N * 2, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(x)
    for _ in range(3):
        buf.offset.zero_()
        sp = dense_to_tilesparse(x, None, buf)
        unpack_batch_(sp, out, 0, sp.grid_n, N, M, sp.grid_m * sp.grid_n)
    torch.cuda.synchronize()
    if not torch.equal(out, x):
        raise RuntimeError("round trip mismatch")
    print("profile case ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the sweep, MLP and CPU-baseline extras")
    ap.add_argument("--no-train", action="store_true",
                    help="skip the config-5 DP decoder and config-4 token-sharded sections")
    ap.add_argument("--train-only", action="store_true",
                    help="run only the config-5 / config-4 multi-GPU sections")
    ap.add_argument("--sweep-only", action="store_true",
                    help="of the extras run only the sparsity / structure sweep")
    ap.add_argument("--mlp-only", action="store_true",
                    help="run only the sparse-MLP fwd+bwd comparison (configs 2 and 4)")
    ap.add_argument("--gemm-case", action="store_true",
                    help="run only the small ncu capture case of the masked tcgen05 GEMM")
    ap.add_argument("--kernel-case", choices=["fp8", "relu2", "sparse_recon", "dw", "fp8_compress",
                                                  "tile_scaled"],
                    help="run only a small ncu capture case of that kernel and exit")
    ap.add_argument("--profile-case", action="store_true",
                    help="run only the small ncu capture case and exit")
    args = ap.parse_args()
    if args.gemm_case:
        gemm_case()
        return
    if args.profile_case:
        profile_case()
        return
    if args.kernel_case:
        kernel_cases(args.kernel_case)
        return
    if args.mlp_only:
        import torch
        dev = torch.device("cuda", 0)
        print(json.dumps(mlp_suite(dev)), flush=True)
        return
    if args.train_only:
        import torch
        import torch.distributed as dist
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        if world > 1:
            dist.init_process_group("nccl", device_id=dev)
        out = train_suite(dev, world, rank)
        if rank == 0:
            print(json.dumps(out), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
