"""Throughput of the B200 evaluator on Marina's hot path: the batched transformer forward the
PUCT search calls on each leaf minibatch (src/net/mod.rs:290-296, src/search/mod.rs:686).

One step = one forward pass of a batch of synthetic leaf positions (uniform-random legal
playouts of 0-80 plies, encoded as the reference encodes them) through the `small` network
(d_model 512, 12 layers, 8 heads, d_ff 2048, random init N(0, 0.02) seed 0, per-tensor e4m3
weights) on every GPU. The default precision is fp8w: the weights e4m3-quantised per matrix as
the reference's FP8 path quantises them, bf16 activations -- the precision that meets the
north star's parity bounds (e4m3 activations cannot: see tests/test_precision.py). Each GPU holds
a full weight replica and evaluates its own batch (weak scaling, no collective on the data path;
a gloo process group on the host carries only the barrier and the max over ranks).

    python bench.py [--gpus N --steps K --warmup W --batch B --net small|nano --precision fp8w|fp8|bf16|fp8x2]
    python bench.py --impl reference ...   # the reference's CPU backend (its C restatement) on host cores

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# DRAM bytes (read + write) of all GEMM launches of one forward pass, per position: ncu
# dram__bytes_read.sum + dram__bytes_write.sum summed over the 49 GEMM launches of one pass of
# `bench.py --batch 4096` (fp8w), and of `bench.py --batch 1024 --precision fp8` for fp8. Traffic of
# one full pass = this x the batch.
GEMM_DRAM_BYTES_PER_EVAL = {("small", "fp8w"): 13.84e6, ("small", "fp8"): 7.60e6}
METRIC = "small-net evals/sec per B200 and 8xB200 at batch 256-8192; PUCT nodes/sec"
UNIT = "evals/s"
L2_BYTES = 126 * 2 ** 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--net", choices=["small", "nano"], default="small")
    ap.add_argument("--batch", type=int, default=4096, help="positions per GPU per step")
    ap.add_argument("--precision", choices=["fp8w", "fp8", "bf16", "fp8x2"], default="fp8w")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fp8-peak", action="store_true",
                    help="skip measuring the e4m3 tensor peak (the roofline then uses 2x the bf16 figure)")
    ap.add_argument("--mode", choices=["step", "sweep", "puct", "wholebox", "gemm"], default="step",
                    help="step: the contract's JSON line; sweep: configs[2] latency/throughput per batch size; "
                         "puct: configs[3] nodes/s of the batched PUCT search; wholebox: configs[4] 1M positions; "
                         "gemm: the four encoder GEMMs of the batch beside cuBLASLt (torch._scaled_mm) on the same shapes")
    ap.add_argument("--roots", type=int, default=32)
    ap.add_argument("--nodes", type=int, default=100_000)
    ap.add_argument("--positions", type=int, default=1 << 20)
    ap.add_argument("--chunk", type=int, default=8192)
    ap.add_argument("--ctx-per-gpu", type=int, default=1,
                    help="wholebox: evaluator contexts per GPU (each takes a shard of every chunk; two overlap "
                         "one shard's copies and launches with the other's kernels)")
    ap.add_argument("--scan", action="store_true", help="puct / wholebox: measure at 1, 2, 4, ... up to --gpus GPUs")
    return ap.parse_args()


def load_net(name: str):
    from marina_b200 import model, weights

    arch = model.Architecture.from_json((ROOT / "marina_b200" / "cards" / f"{name}.json").read_text())
    w = weights.random_init(arch, seed=0)
    return arch, w


def workload_config(args, n_gpus: int) -> dict:
    return {
        "workload": f"{args.net} net forward (configs[1] network: d512 L12 8x64 ff2048, e4m3 per-tensor weights)"
        if args.net == "small" else "nano net forward (d192 L6 6x32 ff768)",
        "net": args.net,
        "batch_per_gpu": args.batch,
        "global_batch": args.batch * n_gpus,
        "tokens_per_position": 65,
        "precision": args.precision,
        "parallelism": f"replicas{n_gpus} (no collective)",
        "inputs": "uniform-random legal playouts, 0-80 plies, per-rank seed",
        "l2": "activations (>1 GB per step) exceed the 126 MB L2; a 256 MiB buffer is also rewritten between timed steps",
    }


def algorithmic_bytes(arch, precision: str, positions: int) -> dict:
    """DRAM bytes one pass's kernels of each memory-bound class must move at the layer-boundary
    design: LayerNorm reads the f16 residual row and writes the GEMM operand row (2L - 1 launches);
    attention reads Q, K, V (bf16) and writes its output row (L launches); the embedding writes x
    and layer 0's h; the heads read the 65 rows of x, the legal slots and write the priors and the
    value head's input."""
    d, L, t = arch.d_model, arch.n_layers, arch.tokens
    ab = 1 if precision == "fp8" else 2
    rows = positions * t
    return {"layernorm": (2 * L - 1) * rows * (2 * d + d * ab), "attention": L * rows * (6 * d + d * ab),
            "embed": rows * (2 * d + d * ab) + positions * 66,
            "heads": positions * (t * 2 * d + 224 * 4 * 2 + 2 * d)}


def flops_per_eval(arch) -> float:
    d, ff, t, L = arch.d_model, arch.d_ff, arch.tokens, arch.n_layers
    return 2.0 * t * L * (4 * d * d + 2 * d * ff)


# ---- CPU baseline: the oracle (C restatement of src/net/cpu.rs) on the host cores ---------
def cpu_baseline(args, arch, w, seconds: float, gpu_evaluate=None) -> dict:
    """The oracle on all host threads over a bounded sample of the workload. With `gpu_evaluate`
    (boards, legal -> priors, wdl through the GPU evaluator), the oracle's outputs for the sample are
    also the checker of the GPU's on the same positions: the returned "parity" holds the north
    star's figures (max |prior| and |WDL| differences over legal slots, max KL, tie-aware and raw
    argmax agreement)."""
    import oracle
    from marina_b200 import chess, weights

    threads = os.cpu_count() or 1
    wq = weights.fp8_weights(w) if args.precision != "bf16" else w
    net = oracle.OracleNetwork(arch, wq, threads=threads)
    # every thread gets at least one 512-row slice (src/net/cpu.rs:352 slices rows the same way)
    chunk = min(max(16 * threads, 16), 2048)
    boards, legal, counts, _ = chess.random_positions(4242, chunk)
    net.evaluate(boards[:2], legal[:2])  # warm
    done, t0 = 0, time.perf_counter()
    while True:
        ref_p, ref_w = net.evaluate(boards, legal)
        done += chunk
        el = time.perf_counter() - t0
        if el >= seconds or el > 0 and done / el * seconds < chunk * 0.5:
            break
    el = time.perf_counter() - t0
    out = {"value": done / el, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": f"{done} positions of the {args.net} config ({chunk}-position batches) in {el:.1f} s"}
    if gpu_evaluate is not None:
        out["parity"] = parity(*gpu_evaluate(boards, legal), ref_p, ref_w, counts)
    return out


def parity(priors, wdl, ref_p, ref_w, counts) -> dict:
    """The north star's parity figures of GPU outputs against the oracle's on the same positions."""
    tie = 2e-4
    n = len(counts)
    prior = max(float(np.abs(priors[p, :c] - ref_p[p, :c]).max()) for p, c in enumerate(counts))
    kl = max(float(np.sum(ref_p[p, :c] * (np.log(np.maximum(ref_p[p, :c], 1e-30))
                                          - np.log(np.maximum(priors[p, :c], 1e-30))))) for p, c in enumerate(counts))
    raw = float(np.mean([np.argmax(priors[p, :c]) == np.argmax(ref_p[p, :c]) for p, c in enumerate(counts)]))
    tied = float(np.mean([ref_p[p, np.argmax(priors[p, :c])] >= ref_p[p, :c].max() - tie
                          for p, c in enumerate(counts)]))
    return {"positions": n, "prior_max_abs": prior, "wdl_max_abs": float(np.abs(wdl - ref_w).max()), "kl_max": kl,
            "argmax_tie_aware": tied, "argmax_raw": raw, "tie": tie,
            "bounds": {"prior": 3e-2, "wdl": 2e-2, "kl": 1e-2, "argmax": 0.99}}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    arch, w = load_net(args.net)
    import oracle
    from marina_b200 import chess, weights

    threads = os.cpu_count() or 1
    wq = weights.fp8_weights(w) if args.precision != "bf16" else w
    net = oracle.OracleNetwork(arch, wq, threads=threads)
    sample = min(max(8 * threads, 16), 2048)
    boards, legal, _, _ = chess.random_positions(4242, sample)
    for _ in range(args.warmup):
        net.evaluate(boards, legal)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        net.evaluate(boards, legal)
    el = time.perf_counter() - t0
    value = sample * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, args.gpus) | {"batch_per_step": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} positions per step of the {args.net} config"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's CPU backend (src/net/cpu.rs) is Rust and no Rust toolchain exists here; "
                "this arm times its C restatement (oracle/) on all host threads",
    }
    print(json.dumps(line), flush=True)


def reduce_max(v: float, world: int) -> float:
    """The maximum of `v` over all ranks of the default (gloo, host) process group (identity when
    alone)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- clocks during the timed region ---------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.lines = device, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, watts, mx, reasons = [], [], None, set()
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
            try:
                watts.append(float(f[3]))
            except ValueError:
                pass
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "power_w": float(np.median(watts)) if watts else None, "samples": len(sm)}


def measure_fp8_peak(dev, seconds: float = 1.5) -> float | None:
    """Sustained dense e4m3 throughput of this GPU in TFLOP/s: cuBLASLt (torch._scaled_mm) on
    8192^3 e4m3 x e4m3 -> bf16, back to back for `seconds`, timed with CUDA events over the last
    two thirds (after the clocks have settled at the power cap). The roofline denominator for the
    FP8 GEMMs, which MEASURED_PEAKS.json does not carry; None if the probe cannot run."""
    import torch

    try:
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        one = torch.tensor(1.0, device=dev)

        def mm():
            return torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)

        for _ in range(3):
            mm()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            mm()
        e1.record()
        torch.cuda.synchronize()
        per = e0.elapsed_time(e1) / 10 / 1e3
        iters = max(10, int(seconds / per))
        for _ in range(iters // 3):
            mm()
        e0.record()
        for _ in range(iters - iters // 3):
            mm()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        return 2.0 * n ** 3 * (iters - iters // 3) / t / 1e12
    except (RuntimeError, AttributeError):
        return None


def run_ours(args):
    import torch
    import torch.distributed as dist

    from marina_b200 import _lib, chess
    from marina_b200.network import B200Network

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        # The ranks share nothing on the data path; a host (gloo) group carries the barrier and
        # the max over ranks of the device timings.
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        return reduce_max(v, world)

    arch, w = load_net(args.net)
    B = args.batch
    net = B200Network(arch, w, device=local, max_batch=B, precision=args.precision)
    boards, legal, counts, _ = chess.random_positions(1 + 1000 * rank, B, 0, 80)
    # A created stream: the events and the forward pass must be ordered on the same stream
    # (the library runs a NULL-stream request on its own non-blocking stream).
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)

    # device-resident inputs / outputs
    d_boards = torch.from_numpy(boards).to(dev)
    d_legal = torch.from_numpy(legal).to(dev)
    d_priors = torch.empty((B, 224), device=dev)
    d_wdl = torch.empty((B, 3), device=dev)
    flush = torch.empty(256 * 2 ** 20 // 4, device=dev)

    def step_device():
        net.evaluate_device(B, d_boards.data_ptr(), d_legal.data_ptr(), d_priors.data_ptr(), d_wdl.data_ptr(),
                            stream.cuda_stream)

    for _ in range(args.warmup):
        step_device()
    torch.cuda.synchronize()
    if net.status_word() != 0:
        raise SystemExit("device fault during warm-up")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step_device()
            ends[i].record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_steps = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = max_over_ranks(float(np.sum(ms_steps)) / args.steps)
    value = world * B / (ms / 1e3)
    if net.status_word() != 0:
        raise SystemExit("device fault during the timed steps")

    # end to end through the public API with pinned host buffers
    h_boards = torch.from_numpy(boards).pin_memory()
    h_legal = torch.from_numpy(legal).pin_memory()
    h_priors = torch.empty((B, 224)).pin_memory()
    h_wdl = torch.empty((B, 3)).pin_memory()
    nb, nl, npr, nw = (t.numpy() for t in (h_boards, h_legal, h_priors, h_wdl))
    for _ in range(max(1, args.warmup)):
        net.evaluate_packed(nb, nl, npr, nw)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        net.evaluate_packed(nb, nl, npr, nw)
    e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
    e2e_value = world * B / e2e_s

    # roofline of the dominant kernel (the GEMM): one eager pass with events around each launch
    prof = net.profile(B, d_boards.data_ptr(), d_legal.data_ptr(), d_priors.data_ptr(), d_wdl.data_ptr(),
                       stream.cuda_stream)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    # The profiled pass runs right after the timed steps (over a second of continuous work, at the
    # power cap), so the sustained cuBLAS figure is the denominator; e4m3 doubles it because the
    # file carries no FP8 figure.
    bf16_peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
    kind = "sustained" if peaks.get("bf16_tflops_sustained") else "burst"
    # fp8x2 issues every e4m3 MMA twice (hi and lo activation terms) at twice the bf16 rate, so its
    # logical FLOPs have the bf16 peak as their ceiling.
    if bf16_peak:
        peak, peak_src = (2 * bf16_peak, f"2x measured bf16 {kind} (MEASURED_PEAKS.json has no fp8 figure)") \
            if args.precision == "fp8" else (bf16_peak, f"measured bf16 {kind} (MEASURED_PEAKS.json)")
    else:
        peak, peak_src = (2 * 1400.0, "2x fallback bf16 sustained") if args.precision == "fp8" \
            else (1400.0, "fallback bf16 sustained")
    peak_2x_bf16 = peak
    fp8_peak = None
    if args.precision == "fp8" and not args.no_fp8_peak:
        fp8_peak = measure_fp8_peak(dev)
        if fp8_peak:
            peak, peak_src = fp8_peak, ("measured here: cuBLASLt e4m3 8192^3 (torch._scaled_mm), sustained "
                                        "over ~1 s at the power cap")
    g = prof["gemm"]
    achieved = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
    traffic = GEMM_DRAM_BYTES_PER_EVAL.get((args.net, args.precision))
    traffic = traffic * B if traffic else None
    total_prof_ms = sum(v["ms"] for v in prof.values())

    launches = net.launches_per_forward(B) * args.steps

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": {"fp8": "e4m3", "fp8w": "bf16", "bf16": "bf16", "fp8x2": "e4m3x2"}[args.precision],
            "data": "synthetic (seeded random-playout positions; random-init weights)",
            "config": workload_config(args, world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic, "traffic_unit": "bytes per pass (DRAM, all GEMM launches)",
                         "kernel": "gemm_tc_kernel (all GEMM launches of one pass)",
                         "peak_source": peak_src, "flops_per_eval": flops_per_eval(arch),
                         "frac_of_2x_bf16": achieved / peak_2x_bf16 if args.precision == "fp8" else None},
            "kernel_ms": {k: round(v["ms"], 4) for k, v in prof.items()},
            "kernel_share": {k: round(v["ms"] / total_prof_ms, 4) for k, v in prof.items()} if total_prof_ms else {},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(B * (66 + 224 * 4)),
                    "d2h_bytes_per_step": int(B * (224 * 4 + 3 * 4 + 4)), "ms_per_step": e2e_s * 1e3,
                    "path": "mrn_evaluate (C ABI) on pinned host buffers: H2D, graph replay, D2H, sync"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "describe": net.describe(),
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args, arch, w, args.cpu_seconds,
                                                gpu_evaluate=lambda b, lg: net.evaluate_packed(b, lg))
            line["config"]["parity"] = line["cpu_baseline"]["parity"]
        print(json.dumps(line), flush=True)
    net.close()
    if world > 1:
        dist.destroy_process_group()


# ---- batch sweep on one GPU ----------------------------------------------------
def run_sweep(args):
    import torch

    from marina_b200 import chess
    from marina_b200.network import B200Network

    arch, w = load_net(args.net)
    sizes = [1, 16, 64, 256, 1024, 4096, 8192]
    net = B200Network(arch, w, device=0, max_batch=max(sizes), precision=args.precision)
    boards, legal, _, _ = chess.random_positions(1, max(sizes), 0, 80)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    d_boards, d_legal = torch.from_numpy(boards).to(dev), torch.from_numpy(legal).to(dev)
    d_priors, d_wdl = torch.empty((max(sizes), 224), device=dev), torch.empty((max(sizes), 3), device=dev)
    pk = peaks()
    bf16_peak = (2 if args.precision == "fp8" else 1) * (pk.get("bf16_tflops_sustained") or 1400.0)
    hbm_peak = pk.get("hbm_gbs") or 6650.0
    for b in sizes:
        step = lambda: net.evaluate_device(b, d_boards.data_ptr(), d_legal.data_ptr(), d_priors.data_ptr(),  # noqa: E731
                                           d_wdl.data_ptr(), stream.cuda_stream)
        for _ in range(args.warmup):
            step()
        times = []
        for _ in range(args.steps):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            step()
            s1.record(stream)
            s1.synchronize()
            times.append(s0.elapsed_time(s1))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            net.evaluate_packed(boards[:b], legal[:b])
        e2e_ms = (time.perf_counter() - t0) / args.steps * 1e3
        net.evaluate_packed_f16(boards[:b], legal[:b])  # the first call allocates its device buffer
        t0 = time.perf_counter()
        for _ in range(args.steps):
            net.evaluate_packed_f16(boards[:b], legal[:b])
        e2e_f16_ms = (time.perf_counter() - t0) / args.steps * 1e3
        prof = net.profile(b, d_boards.data_ptr(), d_legal.data_ptr(), d_priors.data_ptr(), d_wdl.data_ptr(),
                           stream.cuda_stream)
        g = prof["gemm"]
        p50 = float(np.median(times))
        nbytes = algorithmic_bytes(arch, args.precision, b)
        hbm_gbs = {k: round(nbytes[k] / (prof[k]["ms"] / 1e3) / 1e9, 1) for k in nbytes if prof[k]["ms"] > 0}
        print(json.dumps({"mode": "sweep", "net": args.net, "precision": args.precision, "batch": b,
                          "latency_ms_p50": p50, "evals_per_s": b / (p50 / 1e3), "e2e_latency_ms": e2e_ms,
                          "e2e_evals_per_s": b / (e2e_ms / 1e3), "e2e_f16_latency_ms": e2e_f16_ms,
                          "gemm_tflops": g["flops"] / (g["ms"] / 1e3) / 1e12,
                          "gemm_frac_of_bf16_sustained": g["flops"] / (g["ms"] / 1e3) / 1e12 / bf16_peak,
                          "hbm_gbs": hbm_gbs, "hbm_frac": {k: round(v / hbm_peak, 3) for k, v in hbm_gbs.items()},
                          "kernel_ms": {k: round(v["ms"], 4) for k, v in prof.items()}}), flush=True)
    net.close()


def gpu_counts(args) -> list[int]:
    """The GPU counts a puct / wholebox run measures: --gpus alone, or with --scan 1, 2, 4, ... up to it."""
    if not args.scan:
        return [args.gpus]
    out, n = [], 1
    while n < args.gpus:
        out.append(n)
        n *= 2
    return out + [args.gpus]


def peaks() -> dict:
    return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}


# ---- batched PUCT nodes/s on N GPUs (one process, per-GPU evaluator threads) -----
def run_puct(args):
    import ctypes

    from marina_b200 import _lib, chess, search
    from marina_b200.network import B200Network

    arch, w = load_net(args.net)
    workers = 2  # two gathering threads per GPU: one gathers while the other's batch is evaluated
    counts = gpu_counts(args)
    roots_per_worker = -(-args.roots // workers)  # the most any GPU's workers hold (one GPU)
    nets = [B200Network(arch, w, device=g, max_batch=roots_per_worker * 256, precision=args.precision)
            for g in range(max(counts))]
    _, _, _, fens = chess.random_positions(1, args.roots, 0, 80, fens=True)
    roots = [chess.from_fen(f) for f in fens]
    fn = ctypes.cast(_lib.load().mrn_evaluate, ctypes.c_void_p).value
    for n_gpus in counts:
        evaluators = [(fn, net._ctx.value) for net in nets[:n_gpus]]
        search.search(roots[:max(1, 2 * n_gpus)], 2000, evaluators, workers)  # graphs, clocks
        with ClockSampler(0) as clocks:
            per_root, total = search.search(roots, args.nodes, evaluators, workers, search.default_params(256))
        print(json.dumps({"mode": "puct", "net": args.net, "precision": args.precision, "gpus": n_gpus,
                          "roots": args.roots, "node_limit": args.nodes, "leaf_batch": 256,
                          "nodes": total["nodes"], "seconds": total["seconds"],
                          "nodes_per_s": total["nodes"] / total["seconds"],
                          "network_evals": total["network_evals"], "batches": total["batches"],
                          "evals_per_batch": total["network_evals"] / max(1, total["batches"]),
                          "collisions": total["collisions"], "max_depth": total["max_depth"],
                          "workers_per_gpu": workers, "clocks_gpu0": clocks.summary(),
                          "describe": nets[0].describe()}), flush=True)
    for net in nets:
        net.close()


# ---- whole-box throughput, 1M positions in 8192-position chunks over N GPUs -----
def run_wholebox(args):
    """1,048,576 positions in chunks of --chunk positions through the multi-device
    evaluator (`mrn_group_evaluate`: every chunk is cut into one contiguous shard per GPU, evaluated
    at the same time by the library's per-device threads), host buffers pinned. Beside it: the
    fraction of the box's roofline (tensor-bound `small`: GEMM FLOPs at the measured bf16 peak, x2
    for e4m3; HBM-bound `nano`: the layer-boundary bytes at the measured copy bandwidth) and the
    oracle on all host cores on a bounded sample."""
    import torch

    from marina_b200 import chess
    from marina_b200.network import GroupNetwork

    arch, w = load_net(args.net)
    chunk = args.chunk
    t0 = time.perf_counter()
    boards, legal, _, _ = chess.random_positions(1, args.positions, 0, 80)
    gen_s = time.perf_counter() - t0
    hb = torch.from_numpy(boards).pin_memory().numpy()
    hl = torch.from_numpy(legal).pin_memory().numpy()
    hp = torch.empty((args.positions, 224)).pin_memory().numpy()
    hw = torch.empty((args.positions, 3)).pin_memory().numpy()
    pk = peaks()
    bf16 = pk.get("bf16_tflops_sustained") or 1400.0
    gemm_peak = (2 if args.precision == "fp8" else 1) * bf16 * 1e12
    hbm = (pk.get("hbm_gbs") or 6650.0) * 1e9
    d, L, ff, T = arch.d_model, arch.n_layers, arch.d_ff, arch.tokens
    ab = 1 if args.precision == "fp8" else 2
    # layer-boundary algorithmic bytes per position: per layer x (f16) read by 2 LayerNorms and
    # read+written by 2 residual GEMMs; h written by 2 LNs and read by QKV/FFN1; qkv (bf16) written
    # and read; attention out written and read; the FFN hidden written and read.
    bytes_per_eval = T * L * (2 * d * 2 + 2 * 2 * d * 2 + 2 * 2 * d * ab + 2 * 3 * d * 2 + 2 * d * ab + 2 * ff * ab)
    flops = flops_per_eval(arch)
    cpu = cpu_baseline(args, arch, w, args.cpu_seconds) if not args.no_cpu_baseline else None
    for n_gpus in gpu_counts(args):
        devices = [g for g in range(n_gpus) for _ in range(args.ctx_per_gpu)]
        group = GroupNetwork(arch, w, devices, max_batch=chunk, precision=args.precision)
        group.evaluate_packed(hb[:chunk], hl[:chunk], hp[:chunk], hw[:chunk])  # graphs, clocks
        # One call per chunk (each ends when its slowest shard does), then the whole job in one
        # call, which the library runs as the same chunks with no barrier between them.
        t0 = time.perf_counter()
        for a in range(0, args.positions, chunk):
            b = min(a + chunk, args.positions)
            group.evaluate_packed(hb[a:b], hl[a:b], hp[a:b], hw[a:b])
        per_chunk_value = args.positions / (time.perf_counter() - t0)
        with ClockSampler(0) as clocks:
            t0 = time.perf_counter()
            group.evaluate_packed(hb, hl, hp, hw)
            el = time.perf_counter() - t0
        value = args.positions / el
        tensor_frac = value * flops / (n_gpus * gemm_peak)
        hbm_frac = value * bytes_per_eval / (n_gpus * hbm)
        line = {"mode": "wholebox", "net": args.net, "precision": args.precision, "gpus": n_gpus,
                "positions": args.positions, "chunk": chunk, "contexts_per_gpu": args.ctx_per_gpu,
                "seconds": el, "evals_per_s": value, "evals_per_s_one_call_per_chunk": per_chunk_value,
                "roofline": {"bound": "tensor" if args.net == "small" else "hbm",
                             "frac": tensor_frac if args.net == "small" else hbm_frac,
                             "tensor_frac": tensor_frac, "hbm_frac": hbm_frac,
                             "flops_per_eval": flops, "layer_boundary_bytes_per_eval": bytes_per_eval,
                             "peaks": {"gemm_tflops": gemm_peak / 1e12, "hbm_gbs": hbm / 1e9,
                                       "source": "MEASURED_PEAKS.json (bf16 sustained; x2 for e4m3)"}},
                "path": "one mrn_group_evaluate over all positions: chunks of --chunk, shards taken by the "
                        "device threads as they free up (pinned host buffers; per shard: H2D + graph + D2H)",
                "input_generation_s": gen_s, "clocks_gpu0": clocks.summary(), "describe": group.describe()}
        if cpu:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
            line["gpu_over_cpu"] = value / cpu["value"]
        print(json.dumps(line), flush=True)
        group.close()


def run_gemm(args):
    """Our tcgen05 GEMM (through mrn_test_gemm) beside cuBLAS on the encoder's four GEMM shapes at
    this batch: with `--precision fp8` e4m3 operands against cuBLASLt FP8 (torch._scaled_mm, e4m3 x
    e4m3 -> bf16 with a bias; `fp8x2`: ours on two-term e4m3 A, two MMAs per K-step, cuBLASLt on one
    term), otherwise bf16 operands (kind::f16) against cuBLAS bf16
    (torch.addmm). cuBLAS gets the plain bias epilogue on every shape (its residual would be a
    bf16 beta=1 add); ours runs the epilogue the forward pass uses (bias->bf16, GELU->e4m3 or bf16,
    f16 residual add). CUDA events, after warm-up; inputs > L2."""
    import ctypes

    import torch

    from marina_b200 import _lib

    arch, _ = load_net(args.net)
    d, ff, M = arch.d_model, arch.d_ff, args.batch * 65
    dev = torch.device("cuda", 0)
    lib = _lib.load_test()
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    fp8 = args.precision in ("fp8", "fp8x2")
    x2 = args.precision == "fp8x2"  # two-term e4m3 A [M, 2K]; FFN1 writes two-term e4m3 [M, 2N]
    out = []
    for name, N, K, epi, odt in [("qkv", 3 * d, d, 0, torch.bfloat16), ("out_proj", d, d, 3, torch.float16),
                                 ("ffn1", ff, d, 7 if x2 else 2 if fp8 else 1, torch.uint8 if fp8 else torch.bfloat16),
                                 ("ffn2", d, ff, 3, torch.float16)]:
        if fp8:
            a = (torch.randn(M, 2 * K if x2 else K, device=dev) * 0.5).to(torch.float8_e4m3fn)
            b = (torch.randn(N, K, device=dev) * 0.5).to(torch.float8_e4m3fn)
        else:
            a = (torch.randn(M, K, device=dev) * 0.5).to(torch.bfloat16)
            b = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
        bias = torch.randn(N, device=dev)
        ldo = 2 * N if x2 and epi == 7 else N
        o = torch.zeros(M, ldo, device=dev, dtype=odt)

        def ours():
            rc = lib.mrn_test_gemm(2 if x2 else int(fp8), epi, -1, a.data_ptr(), b.data_ptr(), bias.data_ptr(),
                                   o.data_ptr(), ldo, M, N, K, 1e-3 if fp8 else 1.0, 10.0,
                                   ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
            assert rc == 0, lib.mrn_test_last_error().decode()

        one, bias16 = torch.tensor(1.0, device=dev), bias.to(torch.bfloat16)
        a1 = a[:, :K].contiguous() if x2 else a  # cuBLASLt gets one e4m3 term

        def cublas():
            if fp8:
                torch._scaled_mm(a1, b.t(), scale_a=one, scale_b=one, bias=bias16, out_dtype=torch.bfloat16)
            else:
                torch.addmm(bias16, a, b.t())

        row = {"gemm": name, "M": M, "N": N, "K": K}
        for label, fn in (("ours_us", ours), ("cublaslt_us", cublas)):
            for _ in range(max(3, args.warmup)):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            row[label] = e0.elapsed_time(e1) / args.steps * 1e3
        row["ours_tflops"] = 2 * M * N * K / row["ours_us"] / 1e6
        row["cublaslt_tflops"] = 2 * M * N * K / row["cublaslt_us"] / 1e6
        assert int(status.item()) == 0
        out.append(row)
    print(json.dumps({"mode": "gemm", "net": args.net, "batch": args.batch,
                      "dtype": "e4m3x2" if x2 else "e4m3" if fp8 else "bf16",
                      "shapes": out}), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "sweep":
        run_sweep(args)
    elif args.mode == "puct":
        run_puct(args)
    elif args.mode == "wholebox":
        run_wholebox(args)
    elif args.mode == "gemm":
        run_gemm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
