"""Benchmark: sparse-training tokens/s of the byte-level mini-GPT (config 5)
on 1..8 B200 (data parallel, one process per GPU), with the SpMM / SDDMM
roofline of the dominant kernel and the reference's CPU implementation timed
beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Prints ONE JSON line (rank 0).  A "step" is one training step of config 5
on one 32 x 512-token batch per GPU: forward, backward (SDDMM dW + dX on the
cached transpose), values-only gradient all-reduce across ranks, AdamW, and
the SET router step (an update fires every 200 steps).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.abspath(__file__))
METRIC = "SpMM fwd+bwd GB/s vs HBM peak; sparse-train tokens/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seqs", type=int, default=None,
                    help="sequences per CPU sample step (default: the configuration's full batch)")
    ap.add_argument("--kernel", default=None,
                    help="profiling mode: SHAPE:KIND:N runs 2 launches of one kernel "
                         "(SHAPE in %s or MxK@sparsity; KIND fwd|dw|dx|transpose|dtranspose|densegrad, or "
                         "set|rigl for two router updates)" % list(SHAPES))
    ap.add_argument("--workload", choices=["cfg5", "cfg4", "cfg2"], default="cfg5",
                    help="training workload (default cfg5, the headline configuration)")
    ap.add_argument("--graph", action="store_true",
                    help="replay the training step as a CUDA graph (re-captured after "
                         "topology updates); per-kernel timings then come from an eager pass")
    ap.add_argument("--stream", choices=["priority", "default"], default="priority",
                    help="stream for the training step: a high-priority stream (default; the "
                         "weight-gradient SDDMM side stream keeps the lowest priority, so "
                         "critical-path kernels get SMs first) or torch's default stream")
    ap.add_argument("--probe", action="store_true",
                    help="only measure the FP32 and shared-memory ceilings (probe kernels)")
    ap.add_argument("--sweep", action="store_true",
                    help="config-3 standalone SpMM sweep: one JSON line per cell")
    ap.add_argument("--flush", choices=["read", "write"], default="write",
                    help="sweep / kernel timing: L2 flush by reading (default) or writing a "
                         "256 MB buffer between launches")
    ap.add_argument("--sweep-n", default="1,32,256,2048,8192",
                    help="comma-separated N values of the sweep")
    ap.add_argument("--sweep-shapes", default="4096x4096,16384x4096",
                    help="comma-separated MxK shapes of the sweep (config 1 is 256x784)")
    ap.add_argument("--sweep-cpu-max-n", type=int, default=256,
                    help="time the reference's CPU kernels beside the GPU on cells with N up to "
                         "this (0 = never)")
    ap.add_argument("--sweep-sparsity", default="0.5,0.8,0.9,0.95,0.99",
                    help="comma-separated sparsities of the sweep")
    return ap.parse_args()


# Layer shapes of the configs: (M out, K in, sparsity).
SHAPES = {"ffn_up": (3072, 768, 0.9), "ffn_down": (768, 3072, 0.9), "qkv": (2304, 768, 0.7),
          "o": (768, 768, 0.7), "cfg1": (256, 784, 0.9)}


def _shape(spec):
    if spec in SHAPES:
        return SHAPES[spec]
    mk, sp = spec.split("@")
    m, k = mk.lower().split("x")
    return int(m), int(k), float(sp)


def _sweep_matrix(M, K, s, seed=0):
    import sparsecore_b200 as sl

    g = torch.Generator().manual_seed(seed)
    mask = torch.rand(M, K, generator=g) < (1 - s)
    Wd = (torch.randn(M, K, generator=g) * 0.02) * mask
    return sl.PaddedCSR.from_dense(Wd.cuda())


def run_kernel_case(spec):
    """Two launches of one kernel on synthetic inputs (for ncu captures)."""
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    name, kind, n = spec.split(":")
    M, K, s = _shape(name)
    N = int(n)
    W = _sweep_matrix(M, K, s)
    X = torch.randn(K, N, device="cuda")
    dY = torch.randn(M, N, device="cuda")
    WT, _ = sl.transpose_with_perm(W)
    if kind in ("set", "rigl"):
        # one router update on a SparseLinear of this shape (its CSR = W)
        layer = sl.SparseLinear(K, M, bias=False, sparsity=s)
        algo = (sl.SET if kind == "set" else sl.RigL)(sparsity=s, update_freq=1, seed=0)
        layer.apply(algo)
        xin = torch.randn(N, K, device="cuda")
        for _ in range(2):
            layer(xin).square().sum().backward()
            algo.update()
    for _ in range(2 if kind not in ("set", "rigl") else 0):
        if kind == "fwd":
            ops._spmm_raw(W, X)
        elif kind == "dw":
            ops._sddmm_raw(W, dY, X)
        elif kind == "dx":
            ops._spmm_raw(WT, dY)
        elif kind == "densegrad":
            sl.dense_grad(dY, X)
        elif kind == "dtranspose":  # the SparseLinear layout change of an [M, N] activation
            ops._transpose(dY)
        else:
            sl.transpose_with_perm(W)
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": spec, "M": M, "K": K, "N": N, "nnz": W.nnz}))


FLUSH_MODE = {"mode": "write"}


def graph_time_ms(fn, flush_buf, reps=10):
    """Device time of one launch of `fn`: CUDA-graph replay of reps x
    [L2 flush, fn] minus reps x [L2 flush], so neither host launch overhead
    nor a warm L2 enters the number (flush_buf must exceed the L2).  The
    flush overwrites the buffer (mode "write", the default) or reads it
    (mode "read": evicts without leaving dirty lines in L2; measured no
    faster on B200)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    sink = torch.empty((), dtype=flush_buf.dtype, device=flush_buf.device)

    def flush():
        if FLUSH_MODE["mode"] == "write":
            flush_buf.zero_()
        else:
            torch.sum(flush_buf, dim=0, out=sink)

    def capture(with_fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                flush()
                if with_fn:
                    fn()
        return g

    def replay_ms(g):
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(3):
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b))
        return best

    g1, g0 = capture(True), capture(False)
    return max(replay_ms(g1) - replay_ms(g0), 1e-6) / reps


def run_sweep(args):
    """Config 3: W in {4096x4096, 16384x4096} x sparsity x N; fwd, SDDMM, dX."""
    import sparsecore_b200 as sl
    from sparsecore_b200 import _native as N
    from sparsecore_b200 import ops

    hbm, src, sm_max = peaks()
    ceil = N.measure_ceilings()
    fp32 = ceil["fp32_tflops"]
    gather = ceil["gather_ceiling_tflops"]
    print(json.dumps({"measured_ceilings": ceil, "hbm_gbs": hbm, "hbm_source": src}), flush=True)

    flush_buf = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MB > L2

    def t_ms(fn):
        return graph_time_ms(fn, flush_buf)

    shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.sweep_shapes.split(",")]
    if args.sweep_cpu_max_n > 0:
        threads = os.cpu_count() or 1
        os.environ.setdefault("OMP_NUM_THREADS", str(threads))
        print(json.dumps({"cpu": {"threads": threads, "model": cpu_model(),
                                  "method": "reference _core kernels, median of 30 trials "
                                            "(3 above 1 s) after warm-up"}}), flush=True)
    for (M, K) in shapes:
        for s in [float(v) for v in args.sweep_sparsity.split(",")]:
            W = _sweep_matrix(M, K, s)
            WT, _ = sl.transpose_with_perm(W)
            cpu_timer = None  # the reference's CPU kernels on this matrix (built on first use)
            nnz = W.nnz
            for N in [int(v) for v in args.sweep_n.split(",")]:
                if 4 * (K * N + M * N) * 3 > 60e9:
                    continue
                X = torch.randn(K, N, device="cuda")
                dY = torch.randn(M, N, device="cuda")
                cell = {"M": M, "K": K, "sparsity": s, "N": N, "nnz": nnz}
                for kind, fn, byt in (
                        ("fwd", lambda: ops._spmm_raw(W, X), 8 * nnz + 8 * M + 4 * K * N + 4 * M * N),
                        ("dw", lambda: ops._sddmm_raw(W, dY, X), 8 * nnz + 8 * M + 4 * M * N + 4 * K * N),
                        ("dx", lambda: ops._spmm_raw(WT, dY), 8 * nnz + 8 * K + 4 * M * N + 4 * K * N)):
                    ms = t_ms(fn)
                    gbs = byt / (ms * 1e-3) / 1e9
                    tfl = 2 * nnz * N / (ms * 1e-3) / 1e12
                    hbm_floor = byt / (hbm * 1e9) * 1e3
                    fma_floor = 2 * nnz * N / (fp32 * 1e12) * 1e3
                    cell[kind] = {"ms": round(ms, 4), "GB/s": round(gbs, 1),
                                  "hbm_frac": round(gbs / hbm, 3), "TFLOP/s": round(tfl, 2),
                                  "fp32_frac": round(tfl / fp32, 3),
                                  "gather_frac": round(tfl / gather, 3),
                                  "bound": "hbm" if hbm_floor >= fma_floor else "fp32-fma",
                                  "binding_frac": round(max(hbm_floor, fma_floor) / ms, 3)}
                if 0 < N <= args.sweep_cpu_max_n:
                    if cpu_timer is None:
                        from oracle import oracle as O
                        from oracle import ref_arm

                        h = lambda t: t.detach().cpu().numpy().copy()  # noqa: E731
                        p = O.CSR(M, K, h(W.values), h(W.col_indices), h(W.row_start),
                                  h(W.row_nnz), h(W.row_capacity))
                        cpu_timer = ref_arm.KernelTimer(p)
                    ct = cpu_timer.cell(X.cpu().numpy(), dY.cpu().numpy())
                    cell["cpu_ms"] = ct
                    cell["speedup_vs_cpu"] = {k: round(ct[k] / cell[k]["ms"], 1)
                                              for k in ("fwd", "dw", "dx")}
                print(json.dumps(cell), flush=True)
                del X, dY
            del W, WT
            torch.cuda.empty_cache()


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured", float(p.get("sm_max_mhz", 1965.0))
    except Exception:
        return FALLBACK_HBM_GBS, "fallback", 1965.0


def workload_config(wl, world):
    cfg = dict(wl.config)
    cfg["global_batch"] = cfg["global_batch"] * world
    cfg["units_per_step"] = wl.units * world
    cfg["parallelism"] = f"dp{world}"
    cfg["l2"] = "inputs larger than L2 (per-step activations ~GBs, no flush needed)"
    return cfg


# ───────────────────────────── workloads ─────────────────────────────

class Workload:
    """One training configuration: model, router, optimizer, a synthetic batch
    (on the host) and its loss.  `linear` builds the sparse projections (the
    library's SparseLinear on a GPU, the reference kernels on the CPU)."""

    def __init__(self, name, device, rank, linear=None, batch=None, capturable=False):
        import sparsecore_b200 as sl
        from sparsecore_b200 import workloads as W

        self.name = name
        dev = torch.device(device)
        torch.manual_seed(0)  # identical replicas on every rank
        if name in ("cfg5", "cfg4"):
            cfg = W.CFG5 if name == "cfg5" else W.CFG4
            self.cfg = cfg
            self.model = W.MiniGPT(cfg, device=dev, linear=linear)
            if cfg.router == "SET":
                self.algo = sl.SET(sparsity=cfg.ffn_sparsity, drop_fraction=cfg.drop_fraction,
                                   update_freq=cfg.update_freq, seed=0)
            else:
                # X / dY are cloned only before an update step (same topology as
                # cloning every step); under --graph the step keeps one graph
                # with the clones and one without.
                self.algo = sl.RigL(sparsity=cfg.ffn_sparsity, drop_fraction=cfg.drop_fraction,
                                    update_freq=cfg.update_freq, seed=0, capture="update_step")
            self.opt = torch.optim.AdamW(self.model.parameters(), lr=cfg.lr,
                                         capturable=capturable)
            nb = batch or cfg.batch
            self.batch = (W.synthetic_tokens(cfg, nb, seed=1000 + rank),)
            self.units = nb * cfg.seq_len
            self.unit = "tokens/s"
            self.data = "synthetic (uniform random token ids)"
            self.loss_fn = lambda m, b: W.lm_loss(m, b[0])
            self.config = {
                "workload": (f"{cfg.name}: d_model {cfg.d_model}, {cfg.n_layers} layers, "
                             f"{cfg.n_heads} heads, ctx {cfg.seq_len}, vocab {cfg.vocab}, FFN "
                             f"{cfg.d_ff} at {int(cfg.ffn_sparsity * 100)}% / attention "
                             f"projections at {int(cfg.attn_sparsity * 100)}% sparsity (padded "
                             f"CSR, fp32), AdamW {cfg.lr}, {cfg.router} every {cfg.update_freq} "
                             f"steps"),
                "global_batch": cfg.batch, "seq_len": cfg.seq_len}
        else:  # cfg2: MLP 784 -> 512 -> 10, SGD 0.1, SET every 100 steps
            make = linear or (lambda fin, fout, s, bias=True: sl.SparseLinear(fin, fout, bias=bias,
                                                                              sparsity=s, device=dev))
            self.model = torch.nn.Sequential(make(784, 512, 0.9, bias=True), torch.nn.ReLU(),
                                             make(512, 10, 0.9, bias=True))
            self.algo = sl.SET(sparsity=0.9, drop_fraction=0.3, update_freq=100, seed=0)
            self.opt = torch.optim.SGD(self.model.parameters(), lr=0.1)
            nb = batch or 256
            g = torch.Generator().manual_seed(1000 + rank)
            self.batch = (torch.randn(nb, 784, generator=g), torch.randint(0, 10, (nb,), generator=g))
            self.units = nb
            self.unit = "samples/s"
            self.data = "synthetic (x ~ N(0,1), uniform int64 labels)"
            self.loss_fn = lambda m, b: torch.nn.functional.cross_entropy(m(b[0]), b[1])
            self.config = {"workload": "cfg2-mlp: 784->512->10 ReLU, both SparseLinear at 90%, "
                                       "SGD 0.1, SET every 100 steps (drop 0.3)",
                           "global_batch": 256, "seq_len": 1}
        if linear is None:
            self.model.apply(self.algo)

    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.batch)


# ───────────────────────────── clocks ─────────────────────────────

class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms",
                 "200", "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
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


# ───────────────────────────── our arm ─────────────────────────────

def run_ours(args, rank, world, local_rank):
    from sparsecore_b200 import _native as N
    from sparsecore_b200 import ops
    from sparsecore_b200.dist import SparseDataParallel, sync_after_router_step
    from sparsecore_b200.workloads import sparse_live_weights

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.stream == "priority":
        from sparsecore_b200.ops import critical_path_stream

        torch.cuda.set_stream(critical_path_stream(dev))
    ceil = N.measure_ceilings(dev)  # before the workload, on an idle GPU
    wl = Workload(args.workload, dev, rank, capturable=args.graph)
    model, algo, opt = wl.model, wl.algo, wl.opt
    ops.set_async_weight_grad(True)  # the loop below reads .grad after backward()
    # One batched exchange after the backward pass.  (The bucketed exchange
    # overlapped with backward, overlap=True, measured no faster at 2 GPUs:
    # 111.1 vs 110.7 ms per step.)
    ddp = SparseDataParallel(model)
    batch_host = tuple(t.pin_memory() for t in wl.batch)
    batch_dev = tuple(t.to(dev) for t in batch_host)

    ar_events = []  # (start, end) around the gradient exchange, serial pass only

    def train(*batch):
        opt.zero_grad(set_to_none=True)
        loss = wl.loss_fn(model, batch)
        loss.backward()
        if timing_exchange["on"]:
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            ddp.allreduce_grads()
            a1.record()
            ar_events.append((a0, a1))
        else:
            ddp.allreduce_grads()
        opt.step()
        return loss

    timing_exchange = {"on": False}

    def route():
        algo.step()
        sync_after_router_step(ddp, algo)

    def step(batch):
        loss = train(*batch)
        route()
        return loss

    graphed = None
    if args.graph:
        from sparsecore_b200.graph import GraphedStep

        graphed = GraphedStep(model, train, batch_dev,
                              variant=getattr(algo, "graph_variant", None))

        def step(batch):  # noqa: F811 - the graph reads the static batch_dev
            loss = graphed()
            route()
            return loss

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):  # eager (lazy library initialisation happens here)
        train(*batch_dev)
        route()
    if graphed is not None:  # first capture outside the timed region
        graphed.capture()
    barrier()

    timer = ops.KernelTimer()
    clocks = Clocks(local_rank)
    clocks.start()
    l0 = N.launches["count"]
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(s)
    for _ in range(args.steps):
        step(batch_dev)
    e1.record(s)
    barrier()
    launches = N.launches["count"] - l0
    clk = clocks.stop()
    ops.set_kernel_timer(None)
    t_ms = e0.elapsed_time(e1)
    # Per-kernel CUDA-event timings come from a serial eager pass right after
    # the timed region: inside the timed step the weight-gradient SDDMM runs
    # on a side stream, concurrently with the dX kernels, so their event
    # windows would overlap (and graph replay has no per-launch events).
    timed_steps = min(args.steps, 5)
    ops.set_async_weight_grad(False)
    ops.set_kernel_timer(timer)
    timing_exchange["on"] = True
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(timed_steps):
        train(*batch_dev)
    s1.record()
    torch.cuda.synchronize()
    timing_exchange["on"] = False
    serial_ms = s0.elapsed_time(s1) / timed_steps
    exchange_ms = (sum(a.elapsed_time(b) for a, b in ar_events) / len(ar_events)) if ar_events else 0.0
    ops.set_kernel_timer(None)
    ops.set_async_weight_grad(True)
    ksum = timer.summary()

    # end to end: host tokens (pinned) -> device every step, loss read back
    barrier()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        if graphed is not None:
            for d, h in zip(batch_dev, batch_host):
                d.copy_(h, non_blocking=True)
            b = batch_dev
        else:
            b = tuple(t.to(dev, non_blocking=True) for t in batch_host)
        float(step(b).item())
    barrier()
    e2e_ms = (time.perf_counter() - w0) * 1e3

    # one router update + topology broadcast, timed on its own.  RigL needs
    # the captured X / dY of a step first (with capture="update_step" only an
    # update step records them): run one capturing step outside the timing.
    if getattr(algo, "capture", None) == "update_step":
        algo.capture = "every_step"
        train(*batch_dev)
        algo.capture = "update_step"
    barrier()
    r0 = time.perf_counter()
    algo.update()
    ddp.broadcast_topology(0)
    barrier()
    router_ms = (time.perf_counter() - r0) * 1e3

    # Raises if a bounded device-side wait gave up anywhere in the run (its
    # kernel's output would have been incomplete).
    N.check_device_status(dev)

    t = torch.tensor([t_ms, e2e_ms, router_ms, exchange_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, router_ms, exchange_ms = t.tolist()
    if rank != 0:
        return None

    tokens = wl.units * world * args.steps
    hbm, hbm_src, sm_max = peaks()
    dom = max(ksum, key=lambda k: ksum[k]["ms"]) if ksum else None
    roof = None
    if dom:
        d = ksum[dom]
        gbs = d["bytes"] / (d["ms"] * 1e-3) / 1e9
        tfl = d["flops"] / (d["ms"] * 1e-3) / 1e12
        fp32_peak = ceil["fp32_tflops"]
        roof = {"bound": "hbm", "kernel": dom, "achieved": round(gbs, 1), "peak": hbm,
                "unit": "GB/s", "frac": round(gbs / hbm, 4), "peak_source": f"{hbm_src} (MEASURED_PEAKS.json hbm_gbs)",
                "traffic": read_traffic(dom), "launches": d["launches"],
                "avg_launch_ms": round(d["ms"] / d["launches"], 4),
                "achieved_fp32_tflops": round(tfl, 2),
                "fp32_fma_peak_tflops": round(fp32_peak, 1),
                "fp32_frac": round(tfl / fp32_peak, 4),
                "gather_ceiling_tflops": ceil["gather_ceiling_tflops"],
                "gather_frac": round(tfl / ceil["gather_ceiling_tflops"], 4),
                "ceilings": ceil,
                "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 2),
                                "GB/s": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1),
                                "TFLOP/s": round(v["flops"] / (v["ms"] * 1e-3) / 1e12, 2)}
                            for k, v in ksum.items()},
                "step_share": round(sum(v["ms"] for v in ksum.values()) / timed_steps
                                    / serial_ms, 3),
                "serial_ms_per_step": round(serial_ms, 3),
                "kernel_timing": (f"CUDA events around every launch on its stream, serial eager "
                                  f"pass of {timed_steps} steps right after the timed region "
                                  f"(the timed step overlaps the weight-gradient SDDMM with dX "
                                  f"on a side stream)")}
    line = {
        "metric": METRIC, "value": round(tokens / (t_ms * 1e-3), 1), "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": wl.data,
        "config": dict(workload_config(wl, world), sparse_live_weights=sparse_live_weights(model)),
        "roofline": roof,
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": wl.unit,
                "h2d_bytes_per_step": wl.h2d_bytes(),
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "cuda_graph": ({"captures": graphed.captures,
                        "library_launches_per_replay": graphed.launches_per_replay}
                       if graphed is not None else None),
        "clocks": clk,
        "device_status": "clean: no bounded device wait timed out (checked after the run)",
        "gradient_exchange": {
            "bucket_bytes": ddp.bucket_numel * 4,
            "ms_per_step": round(exchange_ms, 3),
            "share_of_step": round(exchange_ms / (t_ms / args.steps), 4),
            "what": ("one pack launch for every sparse layer's live dW slots, one concatenation "
                     "of the dense grads, one NCCL all-reduce (AVG), one unpack launch, one "
                     "multi-tensor copy back; CUDA events around allreduce_grads() in the serial "
                     "pass, max over ranks") if world > 1 else "single GPU: no exchange"},
        "router": {"algorithm": type(algo).__name__, "every_steps": algo.update_freq,
                   "update_plus_broadcast_ms": round(router_ms, 1),
                   "note": "no update falls inside the timed window; amortised cost per step = "
                           "update_plus_broadcast_ms / every_steps"},
    }
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_sample(args.workload, args.cpu_seqs, 1, 2)  # about 25 s at config 5
        cb.pop("_config")
        cb.pop("_data")
        line["cpu_baseline"] = cb
    return line


def read_traffic(kernel):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    try:
        for line in open(path):
            f = line.split()
            if len(f) >= 2 and f[0] == kernel:
                return float(f[1])
    except OSError:
        pass
    return None


# ───────────────────────────── reference arm ─────────────────────────────

def cpu_sample(workload, seqs, warmup, steps, budget_s=None, min_steps=1):
    """The reference's CPU implementation of the path: the same model with
    every sparse projection on the reference's own compiled kernels (OpenMP,
    all host threads) and stock torch CPU ops for the dense parts.  `seqs`
    sequences per step (cfg4/cfg5; None = the configuration's full batch) or
    the full 256-sample batch (cfg2).  With `budget_s`, the timed steps are
    cut to what fits that many seconds at the warm-up step's pace (never
    below `min_steps`).  The result states the steps, warm-up and batch that
    actually ran; nothing is scaled or extrapolated."""
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    torch.set_num_threads(threads)
    from oracle import ref_arm

    kern = ref_arm.kernels()
    wl = Workload(workload, "cpu", 0, linear=ref_arm.linear_factory(kern),
                  batch=seqs if workload != "cfg2" else None)
    model, opt = wl.model, wl.opt

    def step():
        opt.zero_grad(set_to_none=True)
        loss = wl.loss_fn(model, wl.batch)
        loss.backward()
        opt.step()
        return float(loss.item())

    t_step = None
    for _ in range(warmup):
        t0 = time.perf_counter()
        step()
        t_step = time.perf_counter() - t0
    if budget_s is not None and t_step:
        steps = max(min_steps, min(steps, int(budget_s / t_step)))
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    batch = wl.batch[0].shape[0]
    return {"value": round(wl.units * steps / dt, 2), "unit": wl.unit,
            "_config": dict(wl.config, global_batch=batch), "_data": wl.data,
            "cores": threads if kern.kind == "reference" else 1, "kind": kern.kind,
            "steps": steps, "warmup": warmup,
            "sample": f"{steps} timed training steps (after {warmup} warm-up) of the full "
                      f"{workload} batch: {batch} x {wl.units // batch} = {wl.units} "
                      f"{wl.unit.split('/')[0]} per step; reference _core kernels (OpenMP, "
                      f"{threads} threads) + torch CPU dense ops; nothing extrapolated",
            "ms_per_step": round(dt / steps * 1e3, 1)}


# Timed seconds the reference arm may spend (a config-5 step takes about
# 8.5 s on 16 host cores, so the default 20 steps fit).
REFERENCE_BUDGET_S = 200.0


def run_reference(args, rank, world):
    if rank != 0:
        return None
    cb = cpu_sample(args.workload, args.cpu_seqs, max(1, min(args.warmup, 1)), args.steps,
                    budget_s=REFERENCE_BUDGET_S, min_steps=3)
    ref = {"config": cb.pop("_config"), "data": cb.pop("_data")}
    return {
        "metric": METRIC, "impl": "reference", "value": cb["value"], "unit": cb["unit"],
        "n_gpus": world, "steps": cb["steps"], "warmup": cb["warmup"],
        "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": ref["data"],
        "config": dict(ref["config"], parallelism="dp1 (rank 0 on the host cores)"),
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if REPO not in sys.path:
        sys.path.insert(0, REPO)
    if args.kernel:
        run_kernel_case(args.kernel)
        return
    if args.probe:
        from sparsecore_b200 import _native as N

        print(json.dumps({"measured_ceilings": N.measure_ceilings()}), flush=True)
        return
    if args.sweep:
        FLUSH_MODE["mode"] = args.flush
        run_sweep(args)
        return
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        if world > 1:
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
            # One communicator line per rank on stderr (stdout keeps the one
            # JSON line): which rank runs on which GPU over which NCCL.
            probe = torch.ones(1, device=torch.device("cuda", local_rank))
            dist.all_reduce(probe)
            ver = ".".join(str(v) for v in torch.cuda.nccl.version())
            # One write per line, so lines of concurrent ranks do not interleave.
            msg = (f"NCCL communicator: rank {rank} of {world} on cuda:{local_rank} "
                   f"({torch.cuda.get_device_name(local_rank)}), NCCL {ver}, all-reduce check "
                   f"{int(probe.item())} == {world}\n")
            os.write(sys.stderr.fileno(), msg.encode())
        line = run_ours(args, rank, world, local_rank)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
