#!/usr/bin/env python
"""Benchmark of the fgm-kernels quantised GEMM path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE config 1 at the metric's M = 8): the decode GEMM sweep
shapes q 2048x2048, kv 2048x512, o 2048x2048, fused gate/up 2048x16384 and
down 8192x2048 (K x N), int4 weights in the .fgm q4g layout with f16 group-64
scales, over 12 distinct layer copies (~383 MB of weights + scales, larger
than 2x the 126 MB L2, so every step streams its weights from HBM).  A step
is one decode pass through that stack: per layer four activation preps
(attention input, attention output, FFN input, down input; f32 X[8, K] ->
rotate-free quantise + pack) and five GEMMs, i.e. fastgemma's Gemm::run
(forward.rs:128-158) for each projection.  The step is captured once in a
CUDA graph and replayed.

``value`` = weight+scale bytes streamed per step / device time per step
(GB/s).  ``e2e`` = the same metric through the host-pointer C ABI
(fgm_linear_q4g_cuda: pinned host X in, pinned host C out, every call).
``prefill`` = BASELINE config 2 (W8A8, M = 256) in int8 TOPS.
``lm_head`` = BASELINE config 3's int4 LM head (N = 262144, M = 8) split by
output columns over the ranks with an NCCL all-gather of the logits.
``cpu_baseline`` = the reference's own CPU kernels (AMX, else VNNI) on the
host cores over a bounded sample of the same workload.

For N > 1 (torchrun), every rank runs its own copy of the stack (the decode
projections are replicated, not sharded: BASELINE runs them on one GPU), so
the scaling is weak and the step has no collective.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DECODE_SHAPES = [("q", 2048, 2048), ("kv", 2048, 512), ("o", 2048, 2048),
                 ("gate_up", 2048, 16384), ("down", 8192, 2048)]  # (name, K, N)
# which activation feeds each projection: q and kv share the attention input
DECODE_INPUT = {"q": 0, "kv": 0, "o": 1, "gate_up": 2, "down": 3}
PREFILL_SHAPES = [("gate_up", 2048, 16384), ("down", 8192, 2048)]
LM_HEAD_N = 262144
M_DECODE, GROUP, M_PREFILL = 8, 64, 256


def q4g_bytes(k, n, group=GROUP):
    return n * k // 2, (k // group) * n * 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--prefill-copies", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-chain", action="store_true",
                    help="skip the full decode step (BASELINE config 3)")
    ap.add_argument("--chain-context", type=int, default=1024)
    ap.add_argument("--no-lm-head", action="store_true")
    ap.add_argument("--no-config0", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-1 M x shape sweep")
    ap.add_argument("--no-config4", action="store_true")
    ap.add_argument("--config4-ms", default="256,1024,4096",
                    help="config-4 row counts (comma-separated)")
    ap.add_argument("--no-per-call", action="store_true",
                    help="skip the config-1 step timed as per-call launches")
    ap.add_argument("--warm", action="store_true",
                    help="each decode GEMM prefetches the next projection's weights into L2")
    ap.add_argument("--profile-chain", action="store_true",
                    help="only run the config-3 decode step eagerly: two warm-up steps, then one "
                         "inside the NVTX range 'decode_chain' (for ncu launch lists)")
    ap.add_argument("--eager", action="store_true",
                    help="launch the step's kernels directly instead of replaying a CUDA graph "
                         "(same kernels, same order; used for ncu launch lists)")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    HW = 0x8          # HW slowdown
    HW_THERMAL = 0x40
    SW_THERMAL = 0x20
    SW_POWER = 0x4

    def __init__(self, cuda_index: int, period: float = 0.005):
        self.period = period
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            pr = torch.cuda.get_device_properties(cuda_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:  # NVML missing: report no samples rather than guess
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = self.get_reasons(self.h)
                for bit, name in ((self.HW, "hw_slowdown"), (self.HW_THERMAL, "hw_thermal_slowdown"),
                                  (self.SW_THERMAL, "sw_thermal_slowdown"),
                                  (self.SW_POWER, "sw_power_cap")):
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------- CPU reference
def cpu_reference_run(layers: int, seconds: float | None, steps: int | None, warmup: int,
                      seed: int = 7):
    """Time the reference's CPU kernels on this host over the decode workload.

    Returns (GB/s, info).  One sample = one layer of the stack (4 preps +
    5 GEMMs) on layer copy (i % layers), driven by a persistent pool over all
    host cores exactly as fgm-core's Pool does (pool.rs:285-311).
    """
    from oracle.oracle import Oracle, load_reference
    from fastgemma_b200 import fgm_format as F
    import ctypes as C
    impl = load_reference()
    kind = "reference"
    if impl is None:
        impl, kind = Oracle(), "port"
    backend = getattr(impl, "backend", "scalar-port")
    cores = os.cpu_count() or 1
    L = impl.lib
    L.cpu_pool_start(cores, impl.init_fn() if kind == "reference" else None)
    rng = np.random.default_rng(seed)
    xs = {K: rng.standard_normal((M_DECODE, K), dtype=np.float32) for K in (2048, 8192)}
    prep = {}
    for K in (2048, 8192):
        prep[K] = (np.zeros((M_DECODE, K), np.float32), np.zeros((M_DECODE, K), np.int8),
                   np.zeros(M_DECODE, np.float32), np.zeros(16 * K, np.int8))
    ws = []
    for _ in range(layers):
        lw = {}
        for name, K, N in DECODE_SHAPES:
            lw[name] = F.synth_q4g(N, K, GROUP, int(rng.integers(1 << 30)), structured=False)
        ws.append(lw)
    cs = {name: np.zeros((M_DECODE, N), np.float32) for name, K, N in DECODE_SHAPES}
    f_q4g, f_prep = impl.fn("q4g"), impl.fn("prep")
    P = lambda a: a.ctypes.data  # noqa: E731
    per_layer = sum(sum(q4g_bytes(K, N)) for _, K, N in DECODE_SHAPES)

    def one_layer(i):
        lw = ws[i % layers]
        done_inputs = set()
        for name, K, N in DECODE_SHAPES:
            inp = DECODE_INPUT[name]
            rot, qa, qs, pa = prep[K]
            if inp not in done_inputs:
                L.cpu_pool_prep(f_prep, P(xs[K]), K, P(rot), P(qa), P(qs), P(pa), M_DECODE, K, 0)
                done_inputs.add(inp)
            bq, s = lw[name]
            L.cpu_pool_gemm_q4g(f_q4g, M_DECODE, N, K, P(pa), P(qs), P(bq), P(s.view(np.uint16)),
                                GROUP, P(cs[name]), N)

    for i in range(warmup):
        one_layer(i)
    t0 = L.cpu_pool_now()
    n = 0
    while True:
        one_layer(n)
        n += 1
        el = L.cpu_pool_now() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= seconds):
            break
    L.cpu_pool_stop()
    gbs = per_layer * n / el / 1e9
    info = {"kind": kind, "cores": cores, "backend": backend,
            "sample": f"{n} single-layer samples (4 preps + 5 int4 GEMMs, M=8, "
                      f"{per_layer / 1e6:.1f} MB of weights each) rotating over {layers} "
                      f"layer copies, {el:.2f} s"}
    return gbs, el / n, info


def step_config(L):
    """The step both arms time (identical in both lines)."""
    return {"workload": "BASELINE config 1 at M=8: q 2048x2048, kv 2048x512, o 2048x2048, "
                        "gate_up 2048x16384, down 8192x2048 (KxN), int4 q4g group 64 f16 "
                        f"scales, {L} distinct layer copies, 4 preps + 5 GEMMs per layer",
            "weight_bytes_per_step": L * sum(sum(q4g_bytes(K, N)) for _, K, N in DECODE_SHAPES),
            "layers": L, "M": M_DECODE}


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    # one step = the GPU arm's step: every layer of the stack once
    gbs, sec, info = cpu_reference_run(args.layers, None, args.steps * args.layers,
                                       args.warmup * args.layers)
    sec *= args.layers
    line = {
        "metric": "decode W4A8 GEMM weight GB/s (M=8); prefill W8A8 GEMM int8 TOPS at M=256",
        "impl": "reference", "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": step_config(args.layers),
        "execution": {"kernels": "the reference's own CPU kernels (oracle/_ref, built from "
                                 "its sources), every layer of the step once per step",
                      "l2": "the step's weights exceed the host's last-level cache"},
        "cpu_baseline": dict(info, value=gbs, unit="GB/s"),
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU arm
def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return
    import torch
    import torch.distributed as dist
    from fastgemma_b200 import device as D
    from fastgemma_b200 import _lib
    lib = _lib.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if not lib.fgm_cuda_available():
        raise SystemExit("no sm_100 device")

    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    if args.profile_chain:
        step, _, _ = build_decode_chain(dev, gen, args.chain_context)
        step()
        step()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_chain")
        step()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        return
    L = args.layers
    # ---- decode stack: weights streamed from HBM every step
    layers = []
    for _ in range(L):
        lw = {}
        for name, K, N in DECODE_SHAPES:
            wb, sb = q4g_bytes(K, N)
            w = torch.randint(0, 256, (wb,), dtype=torch.uint8, device=dev, generator=gen)
            s = torch.empty((K // GROUP, N), dtype=torch.float32, device=dev).uniform_(
                0.005, 0.02, generator=gen).half()
            lw[name] = (w, s)
        layers.append(lw)
    xs = [torch.randn((M_DECODE, K), dtype=torch.float32, device=dev, generator=gen)
          for K in (2048, 2048, 2048, 8192)]
    wbytes_step = L * sum(sum(q4g_bytes(K, N)) for _, K, N in DECODE_SHAPES)

    # The step as ONE work-list launch: per layer the four preps (each into
    # its own packed buffer) and the five GEMMs, each waiting inside the
    # launch for the prep it reads; every (layer, projection) has its own
    # output rows.
    wl = D.WorkList()
    outs = []
    for l in range(L):
        pidx = []
        for x in xs:
            K = x.shape[1]
            pa, qs = D.packed_a(M_DECODE, K, dev), torch.empty(M_DECODE, device=dev)
            pidx.append((wl.prep(x, K, K, pa, qs), pa, qs))
        for name, K, N in DECODE_SHAPES:
            w, s = layers[l][name]
            ip, pa, qs = pidx[DECODE_INPUT[name]]
            c = torch.empty((M_DECODE, N), dtype=torch.float32, device=dev)
            wl.gemm_q4g(N, K, pa, qs, w, s, GROUP, c, deps=(ip,))
            outs.append(c)
    wl.build(M_DECODE)
    side = torch.cuda.Stream(device=dev)

    def run_step():
        with torch.cuda.stream(side):
            wl.run()

    c0 = lib.fgm_cuda_launch_count()
    run_step()
    launches_per_step = lib.fgm_cuda_launch_count() - c0
    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        time.sleep(0.02)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record(side)
        for _ in range(args.steps):
            run_step()
        e1.record(side)
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / args.steps
    value = world * wbytes_step / (ms * 1e-3) / 1e9
    from fastgemma_b200 import _lib as _L
    _L.call("fgm_cuda_device_status")

    # ---- roofline of the dominant kernel: the work-list kernel is the whole
    # step (one launch), so its launch duration is the step time above.
    # Algorithmic bytes per launch: weights + scales, the preps' f32 rows in
    # and packed rows + scales out, every GEMM's packed rows + scales in and
    # f32 rows out.
    M = M_DECODE
    alg = wbytes_step + L * (sum(M * x.shape[1] * 4 + M * x.shape[1] + M * 4 for x in xs)
                             + sum(M * K + M * 4 + M * N * 4 for _, K, N in DECODE_SHAPES))
    hbm, peak_src = hbm_peak()
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("worklist_config1_M8")
    achieved = alg / (ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic, "peak_source": peak_src,
                "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one ncu "
                                  "capture of this kernel on this list (profiles/"
                                  "worklist_config1_M8.md), not measured in this run",
                "kernel": f"worklist_kernel<MT=1>: {L} layers x (4 preps + 5 int4 GEMMs)",
                "algorithmic_bytes_per_launch": alg, "mean_launch_us": ms * 1e3,
                "launches_timed": args.steps,
                "timing": "CUDA events on the launching stream around the timed steps "
                          "(one launch per step)"}

    # ---- the same step as one launch per prep and per GEMM (the per-call
    # entries in a CUDA graph): what the list replaces
    per_call = None
    if not args.no_per_call:
        per_call = bench_config1_per_call(args, dev, world, layers, xs, side)
    del outs

    # ---- LM head, column-sharded over the ranks
    lm_head = None
    if not args.no_lm_head:
        lm_head = bench_lm_head(args, dev, gen, world, rank)

    # ---- full decode step: every op between the GEMMs too
    chain = None
    if not args.no_chain:
        chain = bench_decode_chain(args, dev, gen, world)

    # ---- prefill: W8A8, M = 256
    prefill = None
    if not args.no_prefill:
        prefill = bench_prefill(args, dev, gen, world)

    # ---- BASELINE config 0 (the metric's own shape), config 1 sweep, config 4
    config0 = bench_config0(args, dev, gen, world) if not args.no_config0 else None
    sweep = bench_config1_sweep(args, dev, gen, world) if not args.no_sweep else None
    config4 = bench_config4(args, dev, world, rank) if not args.no_config4 else None

    # ---- e2e: host buffers in, host results out.  The headline goes through
    # the work list (one call per step); the per-projection drop-in
    # (fgm_linear_q4g_cuda, the reference's call structure) is reported beside it
    e2e = e2e_per_call = None
    if not args.no_e2e:
        e2e = bench_e2e_list(args, world, dev, layers)
        e2e_per_call = bench_e2e(args, world, dev)

    cpu = None
    if not args.no_cpu and rank == 0 and world == 1:
        gbs, _, info = cpu_reference_run(L, args.cpu_seconds, None, 2)
        cpu = dict(info, value=gbs, unit="GB/s")

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "decode W4A8 GEMM weight GB/s (M=8); prefill W8A8 GEMM int8 TOPS at M=256",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded uniform int4 codes, f16 scales U(0.005,0.02), X~N(0,1))",
            "config": step_config(L),
            "execution": {"launch": "one work-list kernel launch per step (fgm_cuda_worklist_run)",
                          "parallelism": f"replicas x{world}",
                          "l2": "inputs larger than L2 "
                                f"({wbytes_step / 1e6:.0f} MB of weights per step > 2 x 126 MB)"},
            "roofline": roofline,
            "config1_per_call": per_call,
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk.summary(),
            "e2e": e2e, "e2e_per_call": e2e_per_call, "prefill": prefill, "lm_head": lm_head, "decode_chain": chain,
            "config0": config0, "config1_sweep": sweep, "config4": config4,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    wl.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _timed(fn, steps, world, dev, stream=None, warm=3):
    """Mean device ms of fn() over `steps` calls, CUDA events on `stream`
    (torch's current stream when None), max over ranks."""
    import torch
    with torch.cuda.stream(stream or torch.cuda.current_stream()):
        for _ in range(warm):
            fn()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = stream or torch.cuda.current_stream()
    with torch.cuda.stream(st):  # fn launches (and graphs replay) on the timed stream
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1), world, dev) / steps


def _all_ranks(flag: bool, world: int, dev) -> bool:
    if world == 1:
        return bool(flag)
    import torch
    import torch.distributed as dist
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def bench_config1_per_call(args, dev, world, layers, xs, side):
    """The config-1 step as separate launches: per layer four prep_rows and
    five gemm_q4g calls (the per-call device entries), captured in one CUDA
    graph -- the launch structure the work list replaces."""
    import torch
    from fastgemma_b200 import device as D
    L, M = len(layers), M_DECODE
    pas = [D.packed_a(M, x.shape[1], dev) for x in xs]
    qss = [torch.empty(M, device=dev) for _ in xs]
    cs = {name: torch.empty((M, N), device=dev) for name, K, N in DECODE_SHAPES}

    def step():
        for l in range(L):
            for i, x in enumerate(xs):
                D.prep_rows(x, x.shape[1], qss[i], pas[i], M, x.shape[1], 0)
            for name, K, N in DECODE_SHAPES:
                w, s = layers[l][name]
                i = DECODE_INPUT[name]
                D.gemm_q4g(M, N, K, pas[i], qss[i], w, s, GROUP, cs[name])

    with torch.cuda.stream(side):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        step()
    ms = _timed(g.replay, max(5, args.steps // 2), world, dev, stream=side)
    del g
    wbytes = L * sum(sum(q4g_bytes(K, N)) for _, K, N in DECODE_SHAPES)
    return {"value": world * wbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "launches_per_step": L * (len(xs) + len(DECODE_SHAPES)),
            "workload": "the config-1 step as 108 launches (prep_rows + gemm_q4g per "
                        "projection) in one CUDA graph"}


def bench_lm_head(args, dev, gen, world, rank):
    """BASELINE config 3's LM head (int4, N = 262144, K = 2048, M = 8) split by
    output columns over the ranks.  Every rank draws the same whole weight and
    X (one seed), keeps its column shard, and -- outside the timed regions --
    checks its gathered logits bit for bit against a whole-width GEMM of the
    same inputs on its own GPU, for the fused path over three calls (both
    double buffers) and for the NCCL path."""
    import torch
    from fastgemma_b200 import device as D
    from fastgemma_b200 import shard as S
    N, K, M = LM_HEAD_N, 2048, M_DECODE
    g = torch.Generator(device=dev)
    g.manual_seed(2718)  # the same weight and X on every rank
    w_full = torch.randint(0, 256, (N * K // 2,), dtype=torch.uint8, device=dev, generator=g)
    s_full = torch.empty((K // GROUP, N), dtype=torch.float32, device=dev).uniform_(
        0.005, 0.02, generator=g).half()
    x = torch.randn((M, K), dtype=torch.float32, device=dev, generator=g)
    nb0, nb1 = S.shard_nblocks(N // 16, world, rank)
    cols = (nb1 - nb0) * 16
    w = w_full[nb0 * 16 * K // 2:nb1 * 16 * K // 2].clone()
    s = s_full[:, nb0 * 16:nb1 * 16].contiguous()
    sh = S.ColumnShardedGemm("q4g", None, None, N, K, GROUP, rank=rank, world=world, device=dev,
                             shard=(w, s))
    pa = D.packed_a(M, K, dev)
    qs = torch.empty(M, dtype=torch.float32, device=dev)
    D.prep_rows(x, K, qs, pa, M, K, 0)
    out = torch.empty((M, N), dtype=torch.float32, device=dev)
    whole = torch.empty((M, N), dtype=torch.float32, device=dev)
    D.gemm_q4g(M, N, K, pa, qs, w_full, s_full, GROUP, whole)  # the parity reference
    steps = max(10, args.steps // 4)

    # launches replayed from CUDA graphs of R calls, so the host's launch rate
    # does not set the pace (the fused call's arguments never change: the
    # kernel counts its calls on the device)
    R = 10
    side = torch.cuda.Stream(device=dev)

    def graphed(fn):
        with torch.cuda.stream(side):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for _ in range(R):
                fn()
        return g

    g_gemm = graphed(lambda: sh.local(M, pa, qs))
    ms_gemm = _timed(g_gemm.replay, steps, world, dev, stream=side) / R
    del g_gemm
    local = sh.local(M, pa, qs)
    ms_gather = _timed(lambda: sh.gather(local, out), steps, world, dev)
    ms_nccl = _timed(lambda: sh(M, pa, qs, out), steps, world, dev)
    out.fill_(float("nan"))
    sh(M, pa, qs, out)
    torch.cuda.synchronize()
    parity_nccl = bool(torch.equal(out.view(torch.int32), whole.view(torch.int32)))
    # the product path: GEMM + all-gather fused in one kernel per rank (NVLink stores)
    shf = S.ColumnShardedGemm("q4g", None, None, N, K, GROUP, rank=rank, world=world, device=dev,
                              shard=(w, s), fused=True, max_rows=M)
    g_fused = graphed(lambda: shf(M, pa, qs))  # R calls: the slots alternate on the device
    ms_step = _timed(g_fused.replay, steps, world, dev, stream=side) / R
    del g_fused
    torch.cuda.synchronize()
    shf._calls = R * (steps + 3) + 1  # the device counted every replayed call (+ the capture warm-up)
    stamps = shf.peers.stamps(dev) if shf.peers is not None else None
    ms_step_eager = _timed(lambda: shf(M, pa, qs), steps, world, dev)
    parity_fused = True
    for _ in range(3):  # consecutive calls alternate the two peer buffers
        res = shf(M, pa, qs)
        torch.cuda.synchronize()
        parity_fused &= bool(torch.equal(res.view(torch.int32), whole.view(torch.int32)))
    # token choice (row argmax of the logits): on the fused path each rank
    # scans the gathered logits; on the NCCL path the ranks exchange only
    # per-row (value, index) pairs
    ms_argmax = _timed(lambda: shf.argmax(M, pa, qs), steps, world, dev)
    tok_ref = whole.argmax(dim=1).to(torch.int32)  # no NaN here: first maximum, as the scan
    tok_f = shf.argmax(M, pa, qs)
    shf.close()
    ms_argmax_pairs = _timed(lambda: sh.argmax(M, pa, qs), steps, world, dev)
    tok_p = sh.argmax(M, pa, qs)
    torch.cuda.synchronize()
    parity_tok = bool(torch.equal(tok_f, tok_ref)) and bool(torch.equal(tok_p, tok_ref))
    parity = _all_ranks(parity_nccl and parity_fused and parity_tok, world, dev)
    wbytes = sum(q4g_bytes(K, N))
    phases = None
    if stamps is not None:  # this rank's last call: own work vs waiting for the others
        t = torch.tensor([stamps["pushed"] - stamps["start"], stamps["arrived"] - stamps["pushed"]],
                         dtype=torch.float64, device=dev)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        phases = {"own_gemm_and_push_us_max": t[0].item() / 1e3,
                  "wait_for_peers_us_max": t[1].item() / 1e3,
                  "source": "%globaltimer stamps of each rank's last graph-replayed call, "
                            "max over ranks"}
    return {"value": wbytes / (ms_step * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_step,
            "ms_per_step_eager": ms_step_eager, "phases": phases,
            "gemm_ms": ms_gemm, "nccl_gather_ms": ms_gather, "nccl_step_ms": ms_nccl,
            "argmax_step_ms": ms_argmax, "argmax_pairs_ms": ms_argmax_pairs,
            "steps": steps, "cols_per_rank": cols,
            "parity": parity,
            "parity_detail": {"fused_3_calls": parity_fused, "nccl": parity_nccl,
                              "tokens": parity_tok, "all_ranks": parity},
            "parity_check": "outside the timed regions, every rank's gathered logits equal a "
                            "whole-width gemm_q4g of the same weight and X on its own GPU, "
                            "bit for bit; tokens equal the whole logits' row argmax",
            "workload": f"BASELINE config 3 LM head: int4 q4g {N}x{K} group {GROUP} f16 scales, "
                        f"M={M}, {world}-way output-column shards; value: one kernel per rank "
                        f"that also stores its columns into every peer's logits over NVLink, "
                        f"{R} calls per CUDA graph replay (gemm_ms likewise; ms_per_step_eager: "
                        f"one host launch per call); "
                        f"nccl_*: the same GEMM followed by an NCCL all-gather (group-32 f32 "
                        f"scales are outside the fgm-kernels format)"}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def int8_peak():
    """(TOPS, source): dense int8 tensor peak.  The measured file holds bf16
    only; int8 runs at twice the bf16 rate on this part, so twice the measured
    bf16 burst figure (nominal dense int8: 4500 TOPS)."""
    pk = _peaks()
    if pk.get("bf16_tflops"):
        return 2.0 * pk["bf16_tflops"], "2 x measured bf16 burst (MEASURED_PEAKS.json)"
    return 2.0 * 1590.0, "2 x fallback bf16 1590 TFLOP/s"


def hbm_peak():
    pk = _peaks()
    if pk.get("hbm_gbs"):
        return pk["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def tc_roofline(ops, bytes_, seconds, gpus=1):
    """Roofline block of an int8 tensor-core GEMM step: achieved TOPS per GPU
    against the int8 peak, and the attainable fraction min(1, AI / ridge)
    with ridge = peak ops / HBM bytes per second."""
    peak, src = int8_peak()
    hbm, _ = hbm_peak()
    ach = ops / seconds / 1e12 / gpus
    ai = ops / bytes_
    ridge = peak * 1e12 / (hbm * 1e9)
    return {"bound": "tensor" if ai >= ridge else "hbm", "achieved": ach, "peak": peak,
            "unit": "TOPS", "frac": ach / peak, "peak_source": src, "ops": ops,
            "algorithmic_bytes": bytes_, "arith_intensity": ai, "ridge": ridge,
            "attainable_frac": min(1.0, ai / ridge)}


def _list_ms(wl, steps, world, dev, stream):
    """Mean device ms of one work-list run (CUDA events on `stream`)."""
    return _timed(lambda: wl.run(stream), steps, world, dev, stream=stream)


def bench_config0(args, dev, gen, world):
    """one decode projection M=8, N=8192, K=2048, int4 g64,
    as fastgemma's Gemm::run -- prep of f32 X then the GEMM -- for 32
    distinct weight copies (285 MB > 2 x L2).  The value runs the 32 (prep,
    GEMM) pairs as one work-list launch; the same pairs as per-call entries
    in one CUDA graph are reported beside it."""
    import torch
    from fastgemma_b200 import device as D
    M, N, K, copies = M_DECODE, 8192, 2048, 32
    wb, sb = q4g_bytes(K, N)
    ws = [(torch.randint(0, 256, (wb,), dtype=torch.uint8, device=dev, generator=gen),
           torch.empty((K // GROUP, N), device=dev).uniform_(0.005, 0.02, generator=gen).half())
          for _ in range(copies)]
    x = torch.randn((M, K), device=dev, generator=gen)
    side = torch.cuda.Stream(device=dev)
    hbm, src = hbm_peak()
    alg = wb + sb + M * K * 4 + M * N * 4

    # one work-list launch: per copy its own prep (into its own packed rows)
    # and the GEMM that waits for it
    wl = D.WorkList()
    outs = []
    for w, s in ws:
        pa, qs = D.packed_a(M, K, dev), torch.empty(M, device=dev)
        ip = wl.prep(x, K, K, pa, qs)
        c = torch.empty((M, N), device=dev)
        wl.gemm_q4g(N, K, pa, qs, w, s, GROUP, c, deps=(ip,))
        outs.append(c)
    wl.build(M)
    ms_list = _list_ms(wl, max(20, args.steps // 4), world, dev, side)
    list_call = ms_list / copies

    # the same pairs as per-call entries, one CUDA graph
    pa, qs = D.packed_a(M, K, dev), torch.empty(M, device=dev)
    c = torch.empty((M, N), device=dev)

    def chain():
        for w, s in ws:
            D.prep_rows(x, K, qs, pa, M, K, 0)
            D.gemm_q4g(M, N, K, pa, qs, w, s, GROUP, c)

    with torch.cuda.stream(side):
        chain()
    torch.cuda.synchronize()
    # parity: the list's last copy equals the per-call entry's output bit for bit
    parity = bool(torch.equal(outs[-1].view(torch.int32), c.view(torch.int32)))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        chain()
    ms = _timed(g.replay, max(5, args.steps // 10), world, dev, stream=side)
    del g
    wl.close()
    per_call = ms / copies
    gbs = (wb + sb) / (list_call * 1e-3) / 1e9
    return {"value": world * gbs, "unit": "GB/s", "us_per_call": list_call * 1e3,
            "frac_hbm": (alg / (list_call * 1e-3) / 1e9) / hbm, "hbm_peak": hbm,
            "peak_source": src, "algorithmic_bytes": alg, "parity_vs_per_call": parity,
            "per_call": {"us_per_call": per_call * 1e3,
                         "weight_gbs": (wb + sb) / (per_call * 1e-3) / 1e9,
                         "frac_hbm": (alg / (per_call * 1e-3) / 1e9) / hbm,
                         "path": "prep_rows + gemm_q4g per copy, one CUDA graph"},
            "workload": f"BASELINE config 0: prep + int4 GEMM M={M} N={N} K={K} g{GROUP} f16 "
                        f"scales, {copies} distinct weight copies per step as one work-list "
                        f"launch (each copy its own prep and output rows); value = weight+"
                        f"scale bytes / (step time / {copies})"}


def bench_config1_sweep(args, dev, gen, world):
    """BASELINE config 1 as fastgemma's gemm_bench sweeps it
    (bench/kernels/gemm_bench.c:253-307): each (M, projection) timed alone
    over distinct weight copies (> 2 x L2 per shape), M in {1, 2, 4, 8, 16},
    prep excluded.  Two forms: the copies' GEMMs as one work-list launch
    (reading rows packed before the run), and the per-call entry back to
    back in one CUDA graph."""
    import torch
    from fastgemma_b200 import device as D
    out = {}
    side = torch.cuda.Stream(device=dev)
    hbm, _ = hbm_peak()
    for name, K, N in DECODE_SHAPES:
        wb, sb = q4g_bytes(K, N)
        copies = max(4, min(128, -(-2 * 126 * 2 ** 20 // (wb + sb))))
        ws = [(torch.randint(0, 256, (wb,), dtype=torch.uint8, device=dev, generator=gen),
               torch.empty((K // GROUP, N), device=dev).uniform_(0.005, 0.02,
                                                                 generator=gen).half())
              for _ in range(copies)]
        c = torch.empty((16, N), device=dev)
        cs = torch.empty((copies, 16, N), device=dev)
        for M in (1, 2, 4, 8, 16):
            x = torch.randn((M, K), device=dev, generator=gen)
            pa, qs = D.packed_a(M, K, dev), torch.empty(M, device=dev)
            D.prep_rows(x, K, qs, pa, M, K, 0)
            alg = wb + sb + M * K + M * 4 + M * N * 4

            wl = D.WorkList()
            for i, (w, s) in enumerate(ws):
                wl.gemm_q4g(N, K, pa, qs, w, s, GROUP, cs[i])
            wl.build(M)
            us_list = _list_ms(wl, 20, world, dev, side) * 1e3 / copies
            wl.close()

            def chain():
                for w, s in ws:
                    D.gemm_q4g(M, N, K, pa, qs, w, s, GROUP, c)

            with torch.cuda.stream(side):
                chain()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                chain()
            ms = _timed(g.replay, 5, world, dev, stream=side)
            del g
            us = ms * 1e3 / copies
            out.setdefault(f"M{M}", {})[name] = {
                "us": us_list, "weight_gbs": (wb + sb) / (us_list * 1e-6) / 1e9,
                "frac_hbm": alg / (us_list * 1e-6) / 1e9 / hbm,
                "per_call_us": us, "per_call_frac_hbm": alg / (us * 1e-6) / 1e9 / hbm}
        del ws, cs
    return {"unit": "us per GEMM / weight GB/s", "results": out,
            "workload": "BASELINE config 1: int4 g64 GEMM alone (prep excluded) over distinct "
                        "weight copies (> 2 x L2 per shape); us/frac_hbm: the copies as one "
                        "work-list launch, us per GEMM = step / copies; per_call_*: "
                        "gemm_q4g back to back in one CUDA graph; frac_hbm = algorithmic "
                        "bytes / time / measured HBM"}


def bench_config4(args, dev, world, rank):
    """M in {256, 1024, 4096} x K=2048 x N=262144 int8
    (the LM-head width), columns sharded over the ranks, NCCL all-gather of
    each rank's column block.  GEMM-only and GEMM + gather are timed apart
    and reported as whole-job int8 TOPS and per-GPU fraction of int8 peak;
    outside the timed regions every rank checks the gathered output bit for
    bit against a whole-width GEMM of the same inputs on its own GPU."""
    import torch
    import torch.distributed as dist
    from fastgemma_b200 import _lib
    from fastgemma_b200 import device as D
    from fastgemma_b200 import shard as S
    lib = _lib.lib()
    N, K = LM_HEAD_N, 2048
    g = torch.Generator(device=dev)
    g.manual_seed(31337)  # same weight on every rank
    w_full = torch.randint(-127, 128, (N * K,), dtype=torch.int8, device=dev, generator=g)
    s_full = torch.empty(N, device=dev).uniform_(0.001, 0.01, generator=g)
    nb0, nb1 = S.shard_nblocks(N // 16, world, rank)
    cols = (nb1 - nb0) * 16
    w = w_full[nb0 * 16 * K:nb1 * 16 * K].clone()
    s = s_full[nb0 * 16:nb1 * 16].contiguous()
    D.q8c_prepare(w, cols, K)
    res = {}
    steps = max(3, args.steps // 20)
    for M in (int(v) for v in args.config4_ms.split(",")):
        x = torch.randn((M, K), device=dev, generator=g)
        qa = torch.empty((M, K), dtype=torch.int8, device=dev)
        qs = torch.empty(M, device=dev)
        pa = D.packed_a(M, K, dev)
        D.prep_rows(x, K, qs, pa, M, K, 0, qa=qa)
        local = torch.empty((M, cols), device=dev)
        gathered = torch.empty((world, M, cols), device=dev)

        def gemm():
            D.gemm_q8c_rows(M, cols, K, qa, qs, w, s, local)

        def gemm_gather():
            gemm()
            if world > 1:
                dist.all_gather_into_tensor(gathered, local)

        # the token choice without the logits gather (engine.rs:297-302): each
        # rank reduces its columns to per-row (value, index) pairs, only the
        # pairs cross NVLink, and every rank merges them
        parts = lib.fgm_cuda_argmax_parts(cols)
        vals = torch.empty((M, parts), device=dev)
        idx = torch.empty((M, parts), dtype=torch.int32, device=dev)
        gv = torch.empty((world, M, parts), device=dev)
        gi = torch.empty((world, M, parts), dtype=torch.int32, device=dev)
        tok = torch.empty(M, dtype=torch.int32, device=dev)

        def gemm_argmax():
            gemm()
            st_ = torch.cuda.current_stream().cuda_stream
            _lib.call("fgm_cuda_argmax_partials", local.data_ptr(), M, cols, cols, nb0 * 16,
                      vals.data_ptr(), idx.data_ptr(), st_)
            if world > 1:
                dist.all_gather_into_tensor(gv, vals)
                dist.all_gather_into_tensor(gi, idx)
                av = gv.permute(1, 0, 2).reshape(M, world * parts).contiguous()
                ai = gi.permute(1, 0, 2).reshape(M, world * parts).contiguous()
            else:
                av, ai = vals, idx
            _lib.call("fgm_cuda_argmax_merge", av.data_ptr(), ai.data_ptr(), M, av.shape[1],
                      tok.data_ptr(), st_)

        ms_gemm = _timed(gemm, steps, world, dev)
        ms_all = _timed(gemm_gather, steps, world, dev)
        ms_tok = _timed(gemm_argmax, steps, world, dev)
        # parity: whole-width GEMM of the same inputs on this GPU
        D.q8c_prepare(w_full, N, K)
        whole = torch.empty((M, N), device=dev)
        D.gemm_q8c_rows(M, N, K, qa, qs, w_full, s_full, whole)
        D.q8c_release(w_full)
        gemm_gather()
        torch.cuda.synchronize()
        ok = True
        for r, (a, b) in enumerate(S.shard_ranges(N // 16, world)):
            src = gathered[r] if world > 1 else local
            ok &= bool(torch.equal(src.view(torch.int32),
                                   whole[:, a * 16:b * 16].contiguous().view(torch.int32)))
        # tokens: the whole logits' row argmax on this GPU
        gemm_argmax()
        wparts = lib.fgm_cuda_argmax_parts(N)
        wv = torch.empty((M, wparts), device=dev)
        wi = torch.empty((M, wparts), dtype=torch.int32, device=dev)
        wt = torch.empty(M, dtype=torch.int32, device=dev)
        st_ = torch.cuda.current_stream().cuda_stream
        _lib.call("fgm_cuda_argmax_partials", whole.data_ptr(), M, N, N, 0, wv.data_ptr(),
                  wi.data_ptr(), st_)
        _lib.call("fgm_cuda_argmax_merge", wv.data_ptr(), wi.data_ptr(), M, wparts,
                  wt.data_ptr(), st_)
        torch.cuda.synchronize()
        ok_tok = bool(torch.equal(tok, wt))
        del whole
        torch.cuda.empty_cache()
        ops = 2.0 * M * N * K
        bytes_ = N * K + N * 4 + world * (M * K + M * 4) + M * N * 4
        res[f"M{M}"] = {
            "gemm_ms": ms_gemm, "gemm_gather_ms": ms_all,
            "gemm_tops": ops / (ms_gemm * 1e-3) / 1e12,
            "gemm_gather_tops": ops / (ms_all * 1e-3) / 1e12,
            "gemm_token_ms": ms_tok, "gemm_token_tops": ops / (ms_tok * 1e-3) / 1e12,
            "roofline_gemm": tc_roofline(ops, bytes_, ms_gemm * 1e-3, world),
            "parity": _all_ranks(ok, world, dev),
            "token_parity": _all_ranks(ok_tok, world, dev)}
        del local, gathered
    D.q8c_release(w)
    return {"unit": "TOPS (whole job)", "results": res, "n_gpus": world,
            "cols_per_rank": cols,
            "workload": f"BASELINE config 4: prep of X~N(0,1) then W8A8 GEMM M x K={K} x N={N}, "
                        f"{world}-way output-column shards (one prepared int8 shard per rank), "
                        f"gather = NCCL all_gather_into_tensor of the [M, N/{world}] blocks "
                        f"(rank-major); gemm_token: the GEMM then the rows' token choice "
                        f"with only (value, index) pairs exchanged (argmax partials per rank, "
                        f"all-gather of the pairs, merge); roofline per GPU; parity: gathered "
                        f"blocks == a whole-width GEMM on each rank's own GPU, bit for bit; "
                        f"token_parity: tokens == the whole logits' row argmax"}


def build_decode_chain(dev, gen, T, L=30, world=1, rank=0):
    """The synthetic config-3 stack on `dev` (random-init weights and caches)
    and its decode step; returns (step, weight bytes per step, extras).
    With world > 1 the layers are replicated and the LM head is
    column-sharded over the ranks: each rank's fused GEMM + NVLink gather
    (fgm_cuda_gemm_q4g_gather) leaves every rank the whole logits, which
    each rank softcaps and scans as at one GPU.  The fused call alternates
    two output slots, counted on the device, so a graph replays the step
    in pairs (extras["calls_per_cycle"] = 2)."""
    import torch
    from fastgemma_b200 import _lib
    from fastgemma_b200 import device as D
    M, H, NH, KVH, HD, FF = M_DECODE, 2048, 8, 2, 256, 8192
    KVD = KVH * HD
    # q, k and v as one [q | k | v] weight, gate and up as one [gate | up]
    # weight: each blob is the weights' n-blocks back to back, so a loader
    # builds it by concatenation, and one GEMM serves the projections that
    # share an input
    QKV = NH * HD + 2 * KVD
    shapes = [("qkv", H, QKV), ("o", NH * HD, H), ("gate_up", H, 2 * FF), ("down", FF, H)]

    def q4(k, n):
        w = torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, device=dev, generator=gen)
        s = torch.empty((k // GROUP, n), device=dev).uniform_(0.005, 0.02, generator=gen).half()
        return w, s

    def norm(n):
        return torch.empty(n, device=dev).uniform_(0.5, 1.5, generator=gen)

    layers = []
    for _ in range(L):
        lw = {name: q4(k, n) for name, k, n in shapes}
        lw.update({nm: norm(n) for nm, n in (("in", H), ("qn", HD), ("kn", HD), ("pa", H),
                                            ("pf", H), ("pff", H))})
        vslots = (T + 3) // 4 * 4
        lw["kc"] = torch.randint(-127, 128, (M, T, KVD), dtype=torch.int8, device=dev,
                                 generator=gen)
        lw["ks"] = torch.empty((M, T), device=dev).uniform_(0.001, 0.02, generator=gen)
        lw["vt"] = torch.randint(-127, 128, (M, vslots * KVD), dtype=torch.int8, device=dev,
                                 generator=gen)
        lw["vs"] = torch.empty((M, T), device=dev).uniform_(0.001, 0.02, generator=gen)
        layers.append(lw)
    lm_w, lm_s = q4(H, LM_HEAD_N)
    sh = None
    if world > 1:  # this rank's column shard of the LM head (n-blocks [nb0, nb1))
        from fastgemma_b200 import shard as S
        nb0, nb1 = S.shard_ranges(LM_HEAD_N // 16, world)[rank]
        kb = H // 64
        w_sh = lm_w[nb0 * kb * 512:nb1 * kb * 512].clone()
        s_sh = lm_s[:, nb0 * 16:nb1 * 16].contiguous()
        sh = S.ColumnShardedGemm("q4g", None, None, LM_HEAD_N, H, GROUP, rank=rank, world=world,
                                 device=dev, shard=(w_sh, s_sh), fused=True, max_rows=M)
    last = {}
    final_norm = norm(H)
    inv_freq = (1.0 / (10000.0 ** (torch.arange(0, HD, 2, device=dev, dtype=torch.float32) / HD)))
    pos = torch.full((M,), T - 1, dtype=torch.int32, device=dev)
    # rope's cos / sin: the host libm table the reference computes per position
    rope_cs = torch.from_numpy(D.rope_table(T, HD, inv_freq.cpu().numpy())).to(dev)
    x = torch.randn((M, H), device=dev, generator=gen)
    f32 = lambda *shape: torch.empty(shape, device=dev)  # noqa: E731
    qkv, attn, o = f32(M, QKV), f32(M, NH * HD), f32(M, H)
    q, k, v = qkv[:, :NH * HD], qkv[:, NH * HD:NH * HD + KVD], qkv[:, NH * HD + KVD:]
    gu, dn = f32(M, 2 * FF), f32(M, H)
    logits = f32(M, LM_HEAD_N)
    pa = {K: D.packed_a(M, K, dev) for K in (H, FF)}
    qs = torch.empty(M, device=dev)
    parts = _lib.lib().fgm_cuda_argmax_parts(LM_HEAD_N)
    avals = torch.empty((M, parts), device=dev)
    aidx = torch.empty((M, parts), dtype=torch.int32, device=dev)
    tok = torch.empty(M, dtype=torch.int32, device=dev)

    x0 = x.clone()
    stream = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731

    def step():
        # glue between the GEMMs runs fused per row: norm_prep = (post-norm,
        # residual add,) pre-norm and prep; qkv_post = head norms, rope and
        # the int8 K / V cache writes; gelu_mul_prep = activation and prep
        x.copy_(x0)  # stands in for the embedding gather
        D.norm_prep(x, None, None, layers[0]["in"], M, H, 1e-6, qs, pa[H])
        for li, lw in enumerate(layers):
            D.gemm_q4g(M, QKV, H, pa[H], qs, lw["qkv"][0], lw["qkv"][1], GROUP, qkv)
            D.qkv_post(q, k, v, M, NH, KVH, HD, lw["qn"], lw["kn"], 1e-6, inv_freq, pos, 0, T,
                       lw["kc"], T * KVD, lw["ks"], T, lw["vt"], lw["vt"].shape[1], lw["vs"], T,
                       q_ld=QKV, kv_ld=QKV, cs=rope_cs)
            D.attend_q8(attn, NH * HD, q, QKV, lw["kc"], T * KVD, lw["ks"], T, lw["vt"],
                        lw["vt"].shape[1], lw["vs"], T, M, NH, KVH, HD, 0, T)
            D.prep_rows(attn, NH * HD, qs, pa[H], M, NH * HD, 0)
            D.gemm_q4g(M, H, NH * HD, pa[H], qs, lw["o"][0], lw["o"][1], GROUP, o)
            D.norm_prep(x, o, lw["pa"], lw["pf"], M, H, 1e-6, qs, pa[H])
            D.gemm_q4g(M, 2 * FF, H, pa[H], qs, lw["gate_up"][0], lw["gate_up"][1], GROUP, gu)
            D.gelu_mul_prep(gu, gu[:, FF:], M, FF, qs, pa[FF], ld=2 * FF)
            D.gemm_q4g(M, H, FF, pa[FF], qs, lw["down"][0], lw["down"][1], GROUP, dn)
            nxt = layers[li + 1]["in"] if li + 1 < L else final_norm
            D.norm_prep(x, dn, lw["pff"], nxt, M, H, 1e-6, qs, pa[H])
        if sh is None:
            D.gemm_q4g(M, LM_HEAD_N, H, pa[H], qs, lm_w, lm_s, GROUP, logits)
            lg = logits
        else:  # this rank's columns, gathered from every rank over NVLink
            lg = sh.fused_call(M, pa[H], qs, stream=torch.cuda.current_stream())
        D.softcap(lg, M, LM_HEAD_N, 30.0)
        _lib.call("fgm_cuda_argmax_partials", lg.data_ptr(), M, LM_HEAD_N, LM_HEAD_N, 0,
                  avals.data_ptr(), aidx.data_ptr(), stream())
        _lib.call("fgm_cuda_argmax_merge", avals.data_ptr(), aidx.data_ptr(), M, parts,
                  tok.data_ptr(), stream())
        last["logits"] = lg

    def whole_tokens():
        """The step's LM head as one whole-width GEMM on this rank from the
        same final packed rows, softcapped and scanned: (logits, tokens)."""
        D.gemm_q4g(M, LM_HEAD_N, H, pa[H], qs, lm_w, lm_s, GROUP, logits)
        D.softcap(logits, M, LM_HEAD_N, 30.0)
        wt = torch.empty(M, dtype=torch.int32, device=dev)
        _lib.call("fgm_cuda_argmax_partials", logits.data_ptr(), M, LM_HEAD_N, LM_HEAD_N, 0,
                  avals.data_ptr(), aidx.data_ptr(), stream())
        _lib.call("fgm_cuda_argmax_merge", avals.data_ptr(), aidx.data_ptr(), M, parts,
                  wt.data_ptr(), stream())
        return logits, wt

    # per-rank weight bytes of one step (the LM head's share only)
    lm_bytes = sum(q4g_bytes(H, LM_HEAD_N)) * (1.0 if sh is None else sh.cols / LM_HEAD_N)
    wbytes = L * sum(sum(q4g_bytes(k_, n_)) for _, k_, n_ in shapes) + lm_bytes
    extras = {"tok": tok, "last": last, "whole_tokens": whole_tokens, "shard": sh,
              "calls_per_cycle": 1 if sh is None else 2}
    return step, wbytes, extras


def bench_decode_chain(args, dev, gen, world):
    """one decode step of a Gemma-E2B-shaped stack for 8
    sequences -- 30 layers (hidden 2048, 8 query heads and 2 KV heads of
    dim 256, MLP 8192), every projection int4 q4g, then the int4 LM head
    (262144 x 2048) and the token choice -- with all the operations between
    the GEMMs (forward.rs:469-654): norms, per-head q/k/v norms, rope, int8
    KV-cache writes, the int8-KV attention over `--chain-context` positions,
    gelu_mul, residual adds, final softcap.  Random-init weights, synthetic
    caches.  At N > 1 GPUs the step is ONE step across the N ranks: the 30
    layers are replicated (every rank holds the same seeded model and rows)
    and the LM head is column-sharded, fused with its NVLink gather; the
    tokens then equal those of one GPU, which the line reports for
    comparison.  The graph holds `calls_per_cycle` steps (two when the fused
    gather alternates its slots)."""
    import torch
    from fastgemma_b200 import _lib
    L, M, T = 30, M_DECODE, args.chain_context
    rank = torch.distributed.get_rank() if world > 1 else 0
    cgen = torch.Generator(device=dev)
    cgen.manual_seed(4321)  # the same model and rows on every rank
    step, wbytes, ex = build_decode_chain(dev, cgen, T, L, world=world, rank=rank)
    per = ex["calls_per_cycle"]
    side = torch.cuda.Stream(device=dev)
    lib = _lib.lib()
    with torch.cuda.stream(side):
        c0 = lib.fgm_cuda_launch_count()
        step()
        ours = lib.fgm_cuda_launch_count() - c0
        for _ in range(2 * per - 1):  # an even number of fused calls before the graph
            step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for _ in range(per):
            step()
    with torch.cuda.stream(side):
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    cycles = max(5, args.steps // 10)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):
        e0.record(side)
        for _ in range(cycles):
            g.replay()
        e1.record(side)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / (cycles * per)
    # outside the timed region: the last step's tokens against the whole-width
    # LM head of the same final rows on this rank (logits bit for bit too)
    tokens = ex["tok"].cpu().tolist()
    got_logits = ex["last"]["logits"].clone()
    with torch.cuda.stream(side):
        whole, wt = ex["whole_tokens"]()
    torch.cuda.synchronize()
    same = bool(torch.equal(got_logits.view(torch.int32), whole.view(torch.int32))
                and wt.cpu().tolist() == tokens)
    parity = _all_ranks(same, world, dev)
    del g
    if ex["shard"] is not None:
        ex["shard"].close()
    return {"value": M / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "weight_gbs_per_gpu": wbytes / (ms * 1e-3) / 1e9, "steps": cycles * per,
            "library_launches_per_step": ours, "context": T, "tokens": tokens,
            "parity": parity,
            "parity_check": "outside the timed region, every rank's LM-head logits of the last "
                            "step (after softcap) and its tokens equal a whole-width gemm_q4g "
                            "of the same final rows on that rank, bit for bit",
            "parallelism": ("one GPU" if world == 1 else
                            f"one step across {world} GPUs: layers replicated, LM head "
                            f"column-sharded {world} ways with the fused NVLink gather"),
            "workload": f"BASELINE config 3: 30 layers (hidden 2048, 8 q heads / 2 KV heads of "
                        f"256, MLP 8192, int4 g64 projections), {M} sequences at context {T}, "
                        f"norms, rope (host libm cos/sin table), int8 KV writes, int8-KV "
                        f"attention, gelu_mul, residuals, int4 LM head 262144 x 2048, softcap, "
                        f"argmax; q|k|v and gate|up as one weight each, the glue between GEMMs "
                        f"fused per row; the same seeded model on every rank; one CUDA graph of "
                        f"{per} step(s) replayed"}


def bench_prefill(args, dev, gen, world):
    import torch
    from fastgemma_b200 import device as D
    copies = args.prefill_copies
    ws = []
    for _ in range(copies):
        lw = {}
        for name, K, N in PREFILL_SHAPES:
            w = torch.randint(-127, 128, (N * K,), dtype=torch.int8, device=dev, generator=gen)
            s = torch.empty(N, dtype=torch.float32, device=dev).uniform_(0.001, 0.01, generator=gen)
            D.q8c_prepare(w, N, K)  # tensor-core operand copy, made once per weight
            lw[name] = (w, s)
        ws.append(lw)
    xs = {K: torch.randn((M_PREFILL, K), dtype=torch.float32, device=dev, generator=gen)
          for _, K, _ in PREFILL_SHAPES}
    pas = {K: D.packed_a(M_PREFILL, K, dev) for K in xs}
    qas = {K: torch.empty((M_PREFILL, K), dtype=torch.int8, device=dev) for K in xs}
    qss = {K: torch.empty(M_PREFILL, dtype=torch.float32, device=dev) for K in xs}
    cs = {name: torch.empty((M_PREFILL, N), dtype=torch.float32, device=dev)
          for name, K, N in PREFILL_SHAPES}

    def step():
        for c in range(copies):
            for name, K, N in PREFILL_SHAPES:
                # quantise (row-major int8 for the tensor cores) then the GEMM
                D.prep_rows(xs[K], K, qss[K], pas[K], M_PREFILL, K, 0, qa=qas[K])
                w, s = ws[c][name]
                D.gemm_q8c_rows(M_PREFILL, N, K, qas[K], qss[K], w, s, cs[name])

    side = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(side):
        step()
    torch.cuda.synchronize()
    if args.eager:
        run = step
    else:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            step()
        run = g.replay
    with torch.cuda.stream(side):
        for _ in range(3):
            run()
    torch.cuda.synchronize()
    steps = max(5, args.steps // 10)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):
        e0.record(side)
        for _ in range(steps):
            run()
        e1.record(side)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / steps
    for lw in ws:  # the tensor-core copies are keyed by the weights' addresses
        for w, _ in lw.values():
            D.q8c_release(w)
    ops = copies * sum(2 * M_PREFILL * N * K for _, K, N in PREFILL_SHAPES)
    # algorithmic bytes: int8 weights + scales, X f32 in, int8 X out of prep and
    # back in, Y f32 out
    bytes_ = copies * sum(N * K + N * 4 + M_PREFILL * K * 4 + 2 * M_PREFILL * K + M_PREFILL * N * 4
                          for _, K, N in PREFILL_SHAPES)
    return {"value": world * ops / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": ms,
            "steps": steps, "roofline": tc_roofline(ops, bytes_, ms * 1e-3),
            "workload": f"BASELINE config 2: M=256 prep + W8A8 GEMM at "
            f"2048x16384 and 8192x2048 (KxN), {copies} weight copies per step"}


def bench_e2e_list(args, world, dev, layers):
    """The config-1 step end to end with host buffers, through
    fgm_cuda_worklist_run; host wall clock per step.  Ways to move the
    step's host data, each timed: the four f32 input matrices either copied
    to the device first (one cudaMemcpyAsync each) or read in place from
    page-locked host memory by the run itself; the outputs either stored by
    the GEMMs straight into page-locked host memory or kept in one device
    block that one cudaMemcpyAsync returns; and the step as 2, 4 or 6 lists of
    consecutive layers, each group's outputs copied back on a second stream
    while the next group runs.  The fastest is the value, the others are
    reported beside it.  Outside the timed region
    every output that reached the host is compared bit for bit with the
    per-call entries (prep_rows + gemm_q4g), for every form."""
    import torch
    from fastgemma_b200 import _lib
    from fastgemma_b200 import device as D
    L, M = len(layers), M_DECODE
    Ks = (2048, 2048, 2048, 8192)
    g = torch.Generator()
    g.manual_seed(99)
    xh = [torch.randn((M, K), generator=g).pin_memory() for K in Ks]
    xd = [torch.empty((M, K), device=dev) for K in Ks]
    out_cols = L * sum(N for _, _, N in DECODE_SHAPES)
    st = torch.cuda.Stream(device=dev)
    wbytes = L * sum(sum(q4g_bytes(K, N)) for _, K, N in DECODE_SHAPES)

    # the per-call reference outputs, computed once on the device
    pa_r = {K: D.packed_a(M, K, dev) for K in set(Ks)}
    qs_r = torch.empty(M, device=dev)
    xs_dev = [h.to(dev) for h in xh]
    refs = []
    for l in range(L):
        for name, K, N in DECODE_SHAPES:
            D.prep_rows(xs_dev[DECODE_INPUT[name]], K, qs_r, pa_r[K], M, K, 0)
            w, s_ = layers[l][name]
            r = torch.empty((M, N), device=dev)
            D.gemm_q4g(M, N, K, pa_r[K], qs_r, w, s_, GROUP, r)
            refs.append(r)
    torch.cuda.synchronize()

    def form(inputs_in_place, outputs_to_host):
        ch = torch.empty((M * out_cols,), dtype=torch.float32).pin_memory()
        cd = None if outputs_to_host else torch.empty((M * out_cols,), device=dev)
        wl = D.WorkList()
        off = 0
        for l in range(L):
            pidx = []
            for x_h, x_d in zip(xh, xd):
                K = x_h.shape[1]
                pa, qs = D.packed_a(M, K, dev), torch.empty(M, device=dev)
                src = x_h if inputs_in_place else x_d
                pidx.append((wl.prep(src, K, K, pa, qs), pa, qs))
            for name, K, N in DECODE_SHAPES:
                w, s = layers[l][name]
                ip, pa, qs = pidx[DECODE_INPUT[name]]
                c = (ch if outputs_to_host else cd)[off:off + M * N].view(M, N)
                off += M * N
                wl.gemm_q4g(N, K, pa, qs, w, s, GROUP, c, deps=(ip,))
        wl.build(M)

        def step():
            with torch.cuda.stream(st):
                if not inputs_in_place:
                    for h, d in zip(xh, xd):
                        d.copy_(h, non_blocking=True)
                wl.run(st)
                if not outputs_to_host:
                    ch.copy_(cd, non_blocking=True)
            st.synchronize()

        for _ in range(max(3, args.warmup)):
            step()
        steps = max(10, args.steps)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        sec = max_over_ranks(time.perf_counter() - t0, world, dev) / steps
        _lib.call("fgm_cuda_device_status")
        ok, o = True, 0
        for r in refs:
            n = r.numel()
            ok &= bool(torch.equal(ch[o:o + n].view(r.shape).to(dev).view(torch.int32),
                                   r.view(torch.int32)))
            o += n
        wl.close()
        return sec, steps, ok

    def pipelined(groups):
        """The step as `groups` work lists of consecutive layers; each group's
        outputs go back on a second stream while the next group runs."""
        ch = torch.empty((M * out_cols,), dtype=torch.float32).pin_memory()
        cd = torch.empty((M * out_cols,), device=dev)
        cs = torch.cuda.Stream(device=dev)
        lists, spans, off = [], [], 0
        for g in range(groups):
            wl = D.WorkList()
            o0 = off
            for l in range(g * L // groups, (g + 1) * L // groups):
                pidx = []
                for x_d in xd:
                    K = x_d.shape[1]
                    pa, qs = D.packed_a(M, K, dev), torch.empty(M, device=dev)
                    pidx.append((wl.prep(x_d, K, K, pa, qs), pa, qs))
                for name, K, N in DECODE_SHAPES:
                    w, s = layers[l][name]
                    ip, pa, qs = pidx[DECODE_INPUT[name]]
                    wl.gemm_q4g(N, K, pa, qs, w, s, GROUP, cd[off:off + M * N].view(M, N),
                                deps=(ip,))
                    off += M * N
            wl.build(M)
            lists.append(wl)
            spans.append((o0, off))
        evs = [torch.cuda.Event() for _ in range(groups)]

        def step():
            with torch.cuda.stream(st):
                for h, d in zip(xh, xd):
                    d.copy_(h, non_blocking=True)
                for wl, ev in zip(lists, evs):
                    wl.run(st)
                    ev.record(st)
            with torch.cuda.stream(cs):
                for (o0, o1), ev in zip(spans, evs):
                    cs.wait_event(ev)
                    ch[o0:o1].copy_(cd[o0:o1], non_blocking=True)
            cs.synchronize()

        for _ in range(max(3, args.warmup)):
            step()
        steps = max(10, args.steps)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        sec = max_over_ranks(time.perf_counter() - t0, world, dev) / steps
        _lib.call("fgm_cuda_device_status")
        ok, o = True, 0
        for r in refs:
            n = r.numel()
            ok &= bool(torch.equal(ch[o:o + n].view(r.shape).to(dev).view(torch.int32),
                                   r.view(torch.int32)))
            o += n
        for wl in lists:
            wl.close()
        return sec, steps, ok

    forms = {}
    for inp in (False, True):
        for outh in (True, False):
            key = ("inputs_read_in_place" if inp else "inputs_copied") + "+" + \
                  ("outputs_stored_to_host" if outh else "outputs_one_copy_back")
            sec, steps, ok = form(inp, outh)
            forms[key] = {"value": world * wbytes / sec / 1e9, "ms_per_step": sec * 1e3,
                          "parity": ok, "steps": steps}
    for groups in (2, 4, 6):
        sec, steps, ok = pipelined(groups)
        forms[f"inputs_copied+{groups}_lists_outputs_copied_back_behind_the_next"] = {
            "value": world * wbytes / sec / 1e9, "ms_per_step": sec * 1e3, "parity": ok,
            "steps": steps}
    best = max(forms, key=lambda k: forms[k]["value"])
    b = forms[best]
    return {"value": b["value"], "unit": "GB/s", "ms_per_step": b["ms_per_step"],
            "h2d_bytes_per_step": sum(M * K * 4 for K in Ks),
            "d2h_bytes_per_step": M * out_cols * 4, "steps": b["steps"],
            "parity": all(f["parity"] for f in forms.values()),
            "path": f"fgm_cuda_worklist_run with page-locked host inputs and outputs "
                    f"({best.replace('+', ', ').replace('_', ' ')}), every output back on the "
                    f"host before the step ends; host wall clock",
            "forms": forms}


def bench_e2e(args, world, dev):
    """Same decode stack through fgm_linear_q4g_cuda with pinned host buffers."""
    import torch
    from fastgemma_b200 import _lib
    from fastgemma_b200 import fgm_format as F
    lib = _lib.lib()
    rng = np.random.default_rng(99)
    L = args.layers
    hw = []
    for _ in range(L):
        lw = {}
        for name, K, N in DECODE_SHAPES:
            bq, s = F.synth_q4g(N, K, GROUP, int(rng.integers(1 << 30)), structured=False)
            _lib.call("fgm_cuda_register", bq.ctypes.data, bq.nbytes)
            _lib.call("fgm_cuda_register", s.ctypes.data, s.nbytes)
            lw[name] = (bq, s)
        hw.append(lw)
    xs = {K: torch.randn((M_DECODE, K), dtype=torch.float32).pin_memory() for K in (2048, 8192)}
    cs = {name: torch.empty((M_DECODE, N), dtype=torch.float32).pin_memory()
          for name, K, N in DECODE_SHAPES}
    h2d = d2h = 0
    for name, K, N in DECODE_SHAPES:
        h2d += L * M_DECODE * K * 4
        d2h += L * M_DECODE * N * 4

    # the caller's buffers are fixed, as in a serving loop: their addresses are
    # taken once, and each step is the 60 library calls alone
    calls = [(xs[K].data_ptr(), K, N, hw[l][name][0].ctypes.data, hw[l][name][1].ctypes.data,
              cs[name].data_ptr()) for l in range(L) for name, K, N in DECODE_SHAPES]
    linear = lib.fgm_linear_q4g_cuda

    def step():
        for xp, K, N, bp, sp, cp in calls:
            rc = linear(xp, K, 0, M_DECODE, N, K, bp, sp, GROUP, cp, N)
            if rc:
                _lib.check(rc)

    for _ in range(max(3, args.warmup // 4)):
        step()
    steps = max(5, args.steps // 10)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    sec = max_over_ranks(time.perf_counter() - t0, world, dev) / steps
    wbytes = L * sum(sum(q4g_bytes(K, N)) for _, K, N in DECODE_SHAPES)
    for l in range(L):
        for bq, s in hw[l].values():
            _lib.call("fgm_cuda_unregister", bq.ctypes.data)
            _lib.call("fgm_cuda_unregister", s.ctypes.data)
    return {"value": world * wbytes / sec / 1e9, "unit": "GB/s", "ms_per_step": sec * 1e3,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "path": "fgm_linear_q4g_cuda per projection (host X in, host C out, synchronous), "
                    "host wall clock"}


if __name__ == "__main__":
    main()
