#!/usr/bin/env python3
"""Benchmark of the B200 gated-scan prefill (NEED's recurrent-scan hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one fused gated scan (sigmoid gates, packed-segment resets, fp32
state, bf16 I/O) over B=16 x T=4096 tokens x C=16*64 channels on each GPU.
Ranks are independent batch shards (weak scaling, no data-path collective).
Device-timed with CUDA events on the launching stream; rank 0 prints one JSON
line with the whole-job tokens/s, the HBM roofline of the scan kernel, the
end-to-end number through the public API (inputs copied from pinned host
memory, outputs read back, every step), the oracle's CPU throughput, and two
side measurements: the T=65536 sequence-parallel scan sharded along T over the
N GPUs (NCCL all-gather of the slice summaries + fix-up), and the ragged
speculative-verify decode step.

``--impl reference`` times the CPU implementation of the same path (the
oracle's C restatement of the reference's chunked scan, all host threads) on a
bounded sample of the workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "scan tokens/s per GPU & % HBM roofline (bf16, T=4096) at 1/2/4/8 B200"
B, T, H, D = 16, 4096, 16, 64
C = H * D
FALLBACK_HBM_GBS = 6650.0
PROFILE = os.path.join(ROOT, "profiles", "gated_scan_bf16_prefill_B16_T4096_C1024.md")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-side", action="store_true", help="skip the sequence-parallel and decode side runs")
    ap.add_argument("--profile", action="store_true",
                    help="only the warm-up and timed steps (for ncu): no clock heat loop, e2e, side runs or CPU leg")
    ap.add_argument("--profile-case", choices=["prefill", "decode", "sp-fixup", "ssd-norm", "ssd-conv", "backward", "assoc", "prologue",
                                               "assoc-step", "assoc-long"],
                    default="prefill",
                    help="with --profile: which kernel's workload to run (one GPU)")
    return ap.parse_args()


def algorithmic_bytes() -> int:
    """Bytes one launch must move: x, decay logit, gate logit read and h written
    (bf16, 8 B per token-channel), the reset mask (1 B per token) and the fp32
    final state."""
    return B * T * C * 2 * 4 + B * T + B * C * 4


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampled every 100 ms while the GPU is loaded."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ helpers
def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """dram bytes per launch from the committed ncu summary, if there is one."""
    try:
        with open(PROFILE) as f:
            m = re.search(r"dram_bytes_per_launch\s*[=:]\s*([0-9]+)", f.read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


def cpu_inputs(rows: int):
    """The prefill workload's first `rows` sequences as the oracle takes them
    (fp32 arrays of bf16-rounded values, uint8 reset mask)."""
    import numpy as np
    import oracle
    from need_b200 import workloads
    rng = np.random.default_rng(0)
    shape = (rows, T, C)
    x = oracle.round_to(rng.standard_normal(shape, dtype=np.float32), "bf16")
    z = oracle.round_to(rng.standard_normal(shape, dtype=np.float32) + np.float32(4.0), "bf16")
    g = oracle.round_to(rng.standard_normal(shape, dtype=np.float32), "bf16")
    seg = workloads.segment_starts(rows, T, seed=0, kind="lognormal", lo=16, hi=4096)
    return x, z, g, seg


CPU_ROWS = B  # the CPU legs time the whole workload: all 16 sequences per step


def cpu_sample_rate(nthreads: int, repeats: int = 3):
    """Oracle (C restatement of the reference's chunked scan) tokens/s on the
    whole prefill workload, all gate math included; median of `repeats` runs."""
    import oracle
    x, z, g, seg = cpu_inputs(CPU_ROWS)
    oracle.gated_scan(x[:1, :256], z[:1, :256], g[:1, :256], seg[:1, :256], dtype="bf16", nthreads=nthreads)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        oracle.gated_scan(x, z, g, seg, dtype="bf16", nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    return CPU_ROWS * T / statistics.median(times), statistics.median(times)


def cpu_sample_text(nthreads: int) -> str:
    return (f"the whole workload per step ({CPU_ROWS} x {T} tokens x {C} channels, bf16-rounded gates, resets); "
            f"C restatement of need_kernels.py:177-226 + the gate math of :330-336, {nthreads} threads "
            f"(work split over (sequence, 64-channel block) in the scan and (sequence, 64-token block) in the gates)")


# ------------------------------------------------------------------ reference arm
def run_reference(args, rank: int):
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    import oracle
    x, z, g, seg = cpu_inputs(CPU_ROWS)
    for _ in range(args.warmup):
        oracle.gated_scan(x, z, g, seg, dtype="bf16", nthreads=nthreads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.gated_scan(x, z, g, seg, dtype="bf16", nthreads=nthreads)
    el = time.perf_counter() - t0
    tps = args.steps * CPU_ROWS * T / el
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(),
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                         "sample": cpu_sample_text(nthreads)},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def workload_config():
    return {"workload": "prefill gated scan: B=16, T=4096, H=16, D=64 (C=1024), bf16 I/O, fp32 state, "
                        "packed-segment resets (lengths lognormal(ln 1024, 0.5) clipped [16, 4096]), "
                        "x~N(0,1), decay logits~N(4,1), input-gate logits~N(0,1)",
            "B": B, "T": T, "H": H, "D": D, "parallelism": "batch-sharded replicas (no collective)",
            "l2": "inputs 403 MB per launch > 126 MB L2: no flush between steps",
            "timing": "device time (CUDA events) of K public gated_scan calls on resident inputs, captured "
                      "in one CUDA graph; direct_calls_ms_per_step times them as back-to-back host calls; "
                      "e2e adds the host copies of every step's inputs and outputs"}


# ------------------------------------------------------------------ our arm
def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from need_b200 import abi
    from need_b200 import need_kernels as nk
    from need_b200 import sp, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    abi.load()  # fails loudly if the library was not built

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.profile and args.profile_case != "prefill":
        profile_side_case(args, dev, nk, sp, workloads)
        return

    w = workloads.prefill(dev, seed=1000 + rank)
    stream = torch.cuda.current_stream(dev)

    def step():
        return nk.gated_scan(w.x, w.z, w.g, seg_start=w.seg, return_final_state=True)

    sampler = ClockSampler(local)
    if not args.profile:
        sampler.start()
    for _ in range(max(args.warmup, 3)):
        step()
    # keep the GPU loaded ~1 s so the clock sampler sees the kernel under load
    torch.cuda.synchronize()
    t_end = time.time() + (0.0 if args.profile else 1.0)
    while time.time() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()

    # The K timed steps are K calls of the public API captured in one CUDA
    # graph: each is a full scan over the same resident inputs, and nothing but
    # the kernels runs between them.  (Back-to-back direct calls are reported
    # beside it: the host's per-call work then adds ~2-4 us of launch gap per
    # step; a one-call graph per step added ~8 us.)
    K = args.steps
    side_stream = torch.cuda.Stream(dev)
    side_stream.wait_stream(stream)
    with torch.cuda.stream(side_stream):
        step()
    stream.wait_stream(side_stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(K):
            step()
    graph.replay()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    barrier()
    ev[0].record(stream)
    graph.replay()
    ev[1].record(stream)
    barrier()
    elapsed_ms = max_over_ranks(ev[0].elapsed_time(ev[1]))
    ms_step = elapsed_ms / K
    value = world * B * T / (ms_step / 1e3)
    launch_ms = ev[0].elapsed_time(ev[1]) / K  # this rank's kernel, one launch per step
    del graph
    # the same K steps as back-to-back direct calls (host work between launches)
    ed = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    barrier()
    ed[0].record(stream)
    for _ in range(K):
        step()
    ed[1].record(stream)
    barrier()
    direct_ms_step = max_over_ranks(ed[0].elapsed_time(ed[1])) / K
    clocks = sampler.stop() if not args.profile else None
    peak, peak_kind = measured_peak()
    achieved = algorithmic_bytes() / (launch_ms / 1e3) / 1e9

    if args.profile:
        if rank == 0:
            print(json.dumps({"profile_run": True, "ms_per_step": ms_step, "avg_launch_ms": launch_ms,
                              "achieved_gbs": achieved}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    # ---------------------------------------------------- end to end, public API
    # Every step copies its inputs in from pinned host memory, runs the public
    # call and copies its result out.  Two input slots and two streams let step
    # k+1's host-to-device copy run while step k's result comes back (PCIe is
    # full duplex); a slot is refilled only after the scan that read it is done.
    pin = lambda t: t.cpu().pin_memory()  # noqa: E731
    hin = (pin(w.x), pin(w.z), pin(w.g), pin(w.seg))
    hout = [torch.empty((B, T, C), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    hfin = [torch.empty((B, C), dtype=torch.float32).pin_memory() for _ in range(2)]
    dbuf = [tuple(torch.empty(t.shape, dtype=t.dtype, device=dev) for t in hin) for _ in range(2)]
    s_in, s_run = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    for ev in ev_free:
        ev.record(s_run)

    def e2e_step(k):
        sl = k % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_free[sl])
            for d, hsrc in zip(dbuf[sl], hin):
                d.copy_(hsrc, non_blocking=True)
            ev_in[sl].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(ev_in[sl])
            dx, dz, dg, ds = dbuf[sl]
            h, hf = nk.gated_scan(dx, dz, dg, seg_start=ds, return_final_state=True)
            ev_free[sl].record(s_run)
            hout[sl].copy_(h, non_blocking=True)
            hfin[sl].copy_(hf, non_blocking=True)

    KE = max(3, min(K, 10))
    for k in range(2):
        e2e_step(k)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for k in range(KE):
        e2e_step(k)
    e1.record(s_run)  # after the last result's copy, which follows every step's copy-in
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / KE
    h2d = sum(t.numel() * t.element_size() for t in hin)
    d2h = hout[0].numel() * hout[0].element_size() + hfin[0].numel() * hfin[0].element_size()
    del hin, hout, hfin, dbuf

    # ---------------------------------------------------- side runs
    side = {}
    if not args.no_side:
        side["sequence_parallel"] = run_sp(dev, world, rank, barrier, max_over_ranks, sp, workloads)
        side["decode_verify"] = run_decode(dev, nk, workloads, barrier, max_over_ranks)
        side["affine_backward"] = run_backward(dev, nk, barrier, max_over_ranks)
        side["segment_starts"] = run_segments(dev, nk, barrier, max_over_ranks)
        side["ssd_prologue"] = run_prologue(dev, nk, barrier, max_over_ranks)
        side["ssd_block"] = run_ssd_block(dev, nk, barrier, max_over_ranks)
        side["assoc_memory"] = run_assoc(dev, nk, barrier, max_over_ranks)
        if world == 1:
            side["reference_gpu"] = run_reference_gpu(dev, nk, workloads)
            side["need_model"] = run_need_model(dev, nk)

    # ---------------------------------------------------- CPU baseline (rank 0, N=1)
    cpu = None
    if rank == 0 and world == 1:
        nthreads = os.cpu_count() or 1
        rate, secs = cpu_sample_rate(nthreads)
        cpu = {"value": rate, "unit": "tokens/s", "cores": nthreads, "kind": "port",
               "sample": cpu_sample_text(nthreads) + f"; median of 3 runs of {secs:.2f} s"}
        ref_cpu = reference_cpu_torch(nthreads)
        if ref_cpu is not None:
            cpu["reference_torch_cpu"] = ref_cpu

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms_step, "direct_calls_ms_per_step": direct_ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": workload_config(),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6.65 TB/s",
                         "traffic": profiled_traffic(), "kernel": "need::scan_kernel<GATED, bf16>",
                         "algorithmic_bytes_per_launch": algorithmic_bytes(),
                         "avg_launch_ms": launch_ms,
                         "frac_of_nominal_8TBs": achieved / 8000.0},
            "e2e": {"value": world * B * T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "api": "need_b200.need_kernels.gated_scan",
                    "pipelining": "two input slots; step k+1 copies in while step k copies out"},
            "gpu_launches": K,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        line.update(side)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_kernels():
    """The reference's own need_kernels module from baseline/_ref (an unmodified
    copy made by baseline/fetch_reference.sh), or None when it is not there."""
    if not os.path.exists(os.path.join(REF_DIR, "need_kernels.py")):
        return None
    sys.dont_write_bytecode = True
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import need_kernels as ref_nk  # noqa: E402  (the reference's module of that name)
    return ref_nk


def run_reference_gpu(dev, nk, workloads):
    """The reference's own GPU code for the same work, on this B200, beside this
    repository's kernels (the reference publishes no numbers of its own):

    * ssd_scan with its Triton kernel (need_kernels.py:119-144, launched at
      :325-329) at NEED's 350M model shape (B=8, T=2048, C=832) and at the
      prefill shape (B=16, T=4096, C=1024), bf16;
    * the headline gated prefill (B=16, T=4096, C=1024 bf16, no resets: the
      reference has none) the way the reference computes it on a GPU: the
      gates as torch ops in bf16 (need_kernels.py:330-336 with a sigmoid
      decay) and affine_recurrence_scan, which on CUDA takes torch's
      associative_scan (need_kernels.py:245-262) or, when that raises, its
      chunked torch scan (:177-226).

    Device time with CUDA events, after a warm-up call (Triton compiles then)."""
    import torch
    ref_nk = reference_kernels()
    if ref_nk is None:
        return {"unavailable": "baseline/_ref holds no copy of the reference (run baseline/fetch_reference.sh)"}
    stream = torch.cuda.current_stream(dev)

    def timed(fn, k, warm=2):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / k

    out = {"triton": bool(ref_nk.HAS_TRITON)}
    g0 = torch.Generator(device=dev).manual_seed(23)
    for name, (Bm, Tm, d) in (("ssd_scan_model_shape", (8, 2048, 832)), ("ssd_scan_prefill_shape", (16, 4096, 1024))):
        xs = [torch.randn(Bm, Tm, d, device=dev, generator=g0).to(torch.bfloat16) for _ in range(5)]
        dskip = torch.full((d,), 0.1, device=dev)
        ref_ms = timed(lambda: ref_nk.ssd_scan(*xs, dskip, 0.001, 0.2), 10)
        our_ms = timed(lambda: nk.ssd_scan(*xs, dskip, 0.001, 0.2), 20)
        out[name] = {"workload": f"ssd_scan B={Bm}, T={Tm}, C={d} bf16",
                     "reference_triton_us": 1e3 * ref_ms, "ours_us": 1e3 * our_ms, "speedup": ref_ms / our_ms}
        del xs
    w = workloads.gated_inputs(B, T, C, z_mean=4.0, dtype=torch.bfloat16, device=dev, seed=24, resets=None)
    path = "associative_scan"
    try:  # the same call the reference makes; it catches a failing associative_scan itself
        scan = ref_nk._get_associative_scan()
        if scan is None:
            path = "chunked torch scan (no associative_scan in this torch)"
        else:
            a = torch.rand(2, 8, 4, device=dev)
            scan(lambda l, r: (r[0] * l[0], r[1] + r[0] * l[1]), (a, a), dim=0)
    except Exception as e:  # noqa: BLE001 -- reported, the reference falls back the same way
        path = f"chunked torch scan (associative_scan raised {type(e).__name__})"

    def reference_gated():
        decay = torch.sigmoid(w.z)
        update = (1.0 - decay) * (torch.sigmoid(w.g) * w.x)
        return ref_nk.affine_recurrence_scan(decay, update, dim=1)

    ref_ms = timed(reference_gated, 3, warm=1)
    our_ms = timed(lambda: nk.gated_scan(w.x, w.z, w.g), 20)
    out["gated_prefill"] = {"workload": "gated scan B=16, T=4096, C=1024 bf16, no resets",
                            "reference_path": f"torch gate ops + affine_recurrence_scan ({path})",
                            "reference_us": 1e3 * ref_ms, "ours_us": 1e3 * our_ms, "speedup": ref_ms / our_ms}
    return out


def run_need_model(dev, nk):
    """NEED's own model at config 5: the ~350M preset (config_for_size.py,
    block_size raised to 2048), seeded N(0, 0.02) weights, eval, bf16 autocast
    (the reference's inference setting), one forward over 8 x 2048 random token
    ids.  Timed on this B200: with the reference's kernels (Triton), with this
    repository's need_kernels bound in their place (every ssd_scan on
    libneed_scan.so), the time the drop-in's 14 scan calls take inside that
    forward (CUDA events around each call), and with every
    StructuredDualRetention.forward replaced by the fused patch (in_proj ->
    ssd_conv_scan with the out_norm -> out)."""
    import torch
    ref_nk = reference_kernels()
    if ref_nk is None:
        return {"unavailable": "baseline/_ref holds no copy of the reference (run baseline/fetch_reference.sh)"}
    import config_for_size  # noqa: E402  (from baseline/_ref)
    import need_core  # noqa: E402
    Bm, Tm = 8, 2048
    cfg, _ = config_for_size.model_config_for_params(350_000_000, block_size=Tm)
    cfg["image_2d_scan"] = False  # not on the kernel path; raises under CUDA autocast
    torch.manual_seed(0)
    with torch.device(dev):
        model = need_core.NeedModel(need_core.NeedConfig(**cfg)).eval()
    g0 = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, model.cfg.vocab_size, (Bm, Tm), device=dev, generator=g0)
    stream = torch.cuda.current_stream(dev)

    def forward():
        with torch.no_grad(), torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            return model(ids)[0]

    def timed(k=5):
        forward()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            forward()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / k

    saved = need_core.need_kernels
    scan_events = []

    class Timed:
        def __getattr__(self, name):
            fn = getattr(nk, name)
            if name != "ssd_scan":
                return fn

            def wrapped(*a, **k):
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record(stream)
                y = fn(*a, **k)
                ev[1].record(stream)
                scan_events.append(ev)
                return y
            return wrapped
    sdr = need_core.StructuredDualRetention
    original = sdr.forward

    def patched(self, x):  # the fused block of the integration notes (no-grad path)
        if torch.is_grad_enabled():
            return original(self, x)
        u, bg, cg, dt, og = self.in_proj(x).chunk(5, dim=-1)
        y = nk.ssd_conv_scan(u, bg, cg, dt, og, self.D, self.cfg.ssd_dt_min, self.cfg.ssd_dt_max,
                             self.dwconv.weight, self.dwconv.bias,
                             norm_weight=self.out_norm.weight, eps=self.out_norm.eps)
        return self.out(y)
    try:
        need_core.need_kernels = ref_nk
        ref_ms = timed()
        need_core.need_kernels = nk
        our_ms = timed()
        sdr.forward = patched
        patched_ms = timed()
        sdr.forward = original
        need_core.need_kernels = Timed()
        forward()
        torch.cuda.synchronize()
        scan_ms = sum(a.elapsed_time(b) for a, b in scan_events)
    finally:
        sdr.forward = original
        need_core.need_kernels = saved
    params = sum(p.numel() for p in model.parameters())
    del model
    return {"workload": f"NeedModel forward, {params / 1e6:.0f}M params (d_model={cfg['d_model']}, "
                        f"{cfg['n_layers']} layers), B={Bm}, T={Tm}, bf16 autocast, random weights",
            "reference_kernels_ms": ref_ms, "drop_in_ms": our_ms,
            "drop_in_tokens_per_s": Bm * Tm / (our_ms / 1e3), "reference_tokens_per_s": Bm * Tm / (ref_ms / 1e3),
            "scan_calls": len(scan_events), "scan_ms": scan_ms, "scan_share": scan_ms / our_ms,
            "fused_block_patch_ms": patched_ms, "fused_block_patch_tokens_per_s": Bm * Tm / (patched_ms / 1e3)}


def reference_cpu_torch(nthreads: int):
    """The reference's own CPU path for the headline workload, on the host
    cores: the gates as torch ops in bf16 and affine_recurrence_scan on CPU
    tensors (need_kernels.py:229-264 -> the chunked scan of :177-226); one
    sequence of the prefill workload (1 x 4096 x 1024, no resets), median of 3."""
    import torch
    ref_nk = reference_kernels()
    if ref_nk is None:
        return None
    torch.set_num_threads(nthreads)
    g = torch.Generator().manual_seed(25)
    x, z, gg = (torch.randn(1, T, C, generator=g).to(torch.bfloat16) for _ in range(3))
    z = (z.float() + 4.0).to(torch.bfloat16)

    def run():
        decay = torch.sigmoid(z)
        return ref_nk.affine_recurrence_scan(decay, (1.0 - decay) * (torch.sigmoid(gg) * x), dim=1)

    run()
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": T / sec, "unit": "tokens/s", "cores": nthreads, "kind": "reference",
            "sample": f"1 of the 16 sequences (1 x {T} tokens x {C} channels, no resets), the reference's "
                      f"torch CPU path, median of 3 runs of {sec:.2f} s"}


def run_sp(dev, world, rank, barrier, max_over_ranks, sp, workloads):
    """T=65536 sequence-parallel scan: B=4, H=32, D=128 bf16, T split over ranks."""
    import torch
    Bs, Ts, Cs = 4, 65536, 32 * 128
    t0, t1 = Ts * rank // world, Ts * (rank + 1) // world
    w = workloads.long_sp(dev, B=Bs, T=Ts, H=32, D=128, seed=7, t_begin=t0, t_end=t1)
    for _ in range(3):
        sp.sp_gated_scan(w.x, w.z, w.g)
    KS = 10
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(KS):
        sp.sp_gated_scan(w.x, w.z, w.g)
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / KS
    byts = Bs * Ts * Cs * 8
    return {"workload": "B=4, T=65536, H=32, D=128 bf16, decay logits~N(5,1), no resets; T split over ranks",
            "tokens_per_s": Bs * Ts / (ms / 1e3), "ms_per_step": ms, "steps": KS,
            "hbm_gbs_per_gpu": byts / world / (ms / 1e3) / 1e9, "scaling": "strong"}


def profile_side_case(args, dev, nk, sp, workloads):
    """One-GPU workloads of the other kernels, for ncu: ``decode`` replays the
    verify + commit graph of 256 sequences x 4 drafted tokens; ``sp-fixup``
    scans the last of 8 slices of the B=4, T=65536, C=4096 workload (the
    deferring local scan of rank 7) and fixes it up, the earlier ranks' maps
    stood in for by its own; ``ssd-norm``
    runs the SSD scan with the RMSNorm kernel after it, ``ssd-conv`` the scan
    with the conv + SiLU folded in (inputs as in-projection chunks) and the
    RMSNorm kernel after it, ``backward`` the reversed-time adjoint scan of the
    affine backward at the prefill shape (B=16, T=4096, C=1024 bf16), ``assoc`` the
    associative memory (feature map + tensor-core kernel) and ``prologue`` the
    conv + SiLU prologue, all at NEED's 350M shape (B=8, T=2048, d_model=832,
    memory_rank=64, bf16); ``assoc-step`` runs the memory's decode step for 256
    sequences."""
    import torch
    if args.profile_case == "prologue":
        g0 = torch.Generator(device=dev).manual_seed(8)
        u = torch.randn(8, 2048, 832, device=dev, generator=g0).to(torch.bfloat16)
        w = (torch.randn(832, 1, 3, device=dev, generator=g0) * 0.5).to(torch.bfloat16)
        b = (torch.randn(832, device=dev, generator=g0) * 0.1).to(torch.bfloat16)
        for _ in range(max(args.warmup, 3) + args.steps):
            nk.ssd_conv_silu(u, w, b)
    elif args.profile_case == "assoc-step":
        g0 = torch.Generator(device=dev).manual_seed(9)
        Ns, r, d = 256, 64, 832
        st = torch.zeros(Ns, r, d, device=dev, dtype=torch.bfloat16)
        dn = torch.zeros(Ns, r, device=dev, dtype=torch.bfloat16)
        qs, ks = torch.randn(Ns, r, device=dev, generator=g0), torch.randn(Ns, r, device=dev, generator=g0)
        vs = torch.randn(Ns, d, device=dev, generator=g0).to(torch.bfloat16)
        for _ in range(max(args.warmup, 3) + args.steps):
            nk.assoc_memory_step(qs, ks, vs, st, dn)
    elif args.profile_case == "backward":  # the affine scan's adjoint, as its autograd backward runs it
        g0 = torch.Generator(device=dev).manual_seed(21)
        shape = (16, 4096, 1024)  # the prefill shape
        decay = torch.sigmoid(torch.randn(shape, device=dev, generator=g0) + 4.0).to(torch.bfloat16)
        g = torch.randn(shape, device=dev, generator=g0).to(torch.bfloat16)
        for _ in range(max(args.warmup, 3) + args.steps):
            nk._affine_adjoint(decay, g, 1)
        torch.cuda.synchronize()
        if nk.workspace_error() != 0:
            raise RuntimeError("a device-side wait gave up")
    elif args.profile_case == "ssd-conv":  # the conv folded into the scan, inputs as in-projection chunks
        g0 = torch.Generator(device=dev).manual_seed(1)
        Bm, Tm, d = 8, 2048, 832
        proj = torch.randn(Bm, Tm, 5 * d, device=dev, generator=g0).to(torch.bfloat16)
        u, bg, cg, dt, og = proj.chunk(5, dim=-1)
        w = (torch.randn(d, 1, 3, device=dev, generator=g0) * 0.5).to(torch.bfloat16)
        b = (torch.randn(d, device=dev, generator=g0) * 0.1).to(torch.bfloat16)
        dskip, nw = torch.full((d,), 0.1, device=dev), torch.ones(d, device=dev)
        for _ in range(max(args.warmup, 3) + args.steps):
            nk.ssd_conv_scan(u, bg, cg, dt, og, dskip, 0.001, 0.2, w, b, norm_weight=nw)
        torch.cuda.synchronize()
        if nk.workspace_error() != 0:
            raise RuntimeError("a device-side wait gave up")
    elif args.profile_case in ("ssd-norm", "assoc"):
        g0 = torch.Generator(device=dev).manual_seed(1)
        Bm, Tm, d = 8, 2048, 832
        xs = [torch.randn(Bm, Tm, d, device=dev, generator=g0).to(torch.bfloat16) for _ in range(5)]
        q = torch.randn(Bm, Tm, 64, device=dev, generator=g0)
        k = torch.randn(Bm, Tm, 64, device=dev, generator=g0)
        dskip, w = torch.full((d,), 0.1, device=dev), torch.ones(d, device=dev)
        for _ in range(max(args.warmup, 3) + args.steps):
            if args.profile_case == "ssd-norm":
                nk.ssd_scan_rms_norm(*xs, dskip, 0.001, 0.2, w, 1e-6)
            else:
                nk.linear_associative_memory(q, k, xs[0])
        torch.cuda.synchronize()
        if nk.workspace_error() != 0:
            raise RuntimeError("a device-side wait gave up")
    elif args.profile_case == "assoc-long":  # one T=16384 sequence: chunk states, their scan, 16 segments
        g0 = torch.Generator(device=dev).manual_seed(1)
        q = torch.randn(1, 16384, 64, device=dev, generator=g0)
        k = torch.randn(1, 16384, 64, device=dev, generator=g0)
        v = torch.randn(1, 16384, 832, device=dev, generator=g0).to(torch.bfloat16)
        for _ in range(max(args.warmup, 3) + args.steps):
            nk.linear_associative_memory(q, k, v)
        torch.cuda.synchronize()
        if nk.workspace_error() != 0:
            raise RuntimeError("a device-side wait gave up")
    elif args.profile_case == "decode":
        w = workloads.verify(dev, N=256, C=1024, k=4, seed=11)
        pool = w.states.clone()
        y, sk = torch.empty_like(w.x), torch.empty_like(w.x)
        for _ in range(max(args.warmup, 3) + args.steps):
            nk.ragged_verify(pool, w.cu_k, (w.z, w.g, w.x), out=(y, sk))
            nk.commit_states(pool, sk, w.cu_k, w.accept)
    else:
        # the last of 8 slices of the sequence-parallel workload (B=4, T=65536,
        # C=4096): its deferring local scan, then its fix-up; the 7 earlier
        # ranks' maps are stood in for by this slice's own (the same
        # statistics), so only one slice is held on the device
        P, T = 8, 65536
        w = workloads.long_sp(dev, B=4, T=T, H=32, D=128, seed=7, t_begin=(P - 1) * T // P, t_end=T)
        last = sp.local_scan(w.x, w.z, w.g, rank=P - 1)
        gathered = torch.stack([last.summary.clone() for _ in range(P)])
        for _ in range(max(args.warmup, 3) + args.steps):
            sp.fixup(last, gathered, P, P - 1)
    torch.cuda.synchronize()
    print(json.dumps({"profile_run": True, "case": args.profile_case}), flush=True)


def run_backward(dev, nk, barrier, max_over_ranks):
    """Backward of affine_recurrence_scan at the prefill shape (B=16, T=4096,
    C=1024, bf16): the reversed-time adjoint scan alone (reads decay and the
    output gradient, writes the update gradient: 6 B per token-channel), and a
    whole scan training step (forward + backward through autograd)."""
    import torch
    g0 = torch.Generator(device=dev).manual_seed(21)
    shape = (B, T, C)
    decay = torch.sigmoid(torch.randn(shape, device=dev, generator=g0) + 4.0).to(torch.bfloat16)
    update = torch.randn(shape, device=dev, generator=g0).to(torch.bfloat16)
    g = torch.randn(shape, device=dev, generator=g0).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, k):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / k

    adj_ms = timed(lambda: nk._affine_adjoint(decay, g, 1), 20)
    d_req, u_req = decay.clone().requires_grad_(True), update.clone().requires_grad_(True)

    def train_step():
        d_req.grad = u_req.grad = None
        nk.affine_recurrence_scan(d_req, u_req).backward(g)

    step_ms = timed(train_step, 10)
    return {"workload": "affine scan backward, B=16, T=4096, C=1024 bf16, decay=sigmoid(N(4,1))",
            "adjoint_ms": adj_ms, "adjoint_hbm_gbs": B * T * C * 6 / (adj_ms / 1e3) / 1e9,
            "fwd_bwd_ms": step_ms, "fwd_bwd_tokens_per_s": B * T / (step_ms / 1e3)}


def run_segments(dev, nk, barrier, max_over_ranks):
    """Reset masks of the prefill's packed windows from int64 token ids
    (B=16, T=4096): reads 8 B and writes 1 B per token; replayed from a CUDA
    graph so that the host's per-call cost is not timed."""
    import torch
    g0 = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(3, 5000, (B, T), device=dev, generator=g0, dtype=torch.int64)
    ids[torch.rand((B, T), device=dev, generator=g0) < 1.0 / 512] = 2  # EOS, ~512-token documents
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)  # warm up off the capture, then replay a graph (device time only)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        nk.segment_starts(ids)
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        nk.segment_starts(ids)
    for _ in range(5):
        graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(100):
        graph.replay()
    e1.record(stream)
    barrier()
    us = 1e3 * max_over_ranks(e0.elapsed_time(e1)) / 100
    return {"workload": "segment starts of B=16 x T=4096 int64 windows", "us_per_call": us,
            "hbm_gbs": B * T * 9 / (us / 1e6) / 1e9}


def run_prologue(dev, nk, barrier, max_over_ranks):
    """The SSD block's conv + SiLU prologue at NEED's model shape (B=8, T=2048,
    C=832, K=3, bf16): the fused kernel (reads 2 B, writes 2 B per element)
    against the same computation as torch ops on the GPU, both replayed from
    CUDA graphs so that the host's per-call cost is not timed."""
    import torch
    import torch.nn.functional as F
    g0 = torch.Generator(device=dev).manual_seed(8)
    Bm, Tm, Cm, K = 8, 2048, 832, 3
    u = torch.randn(Bm, Tm, Cm, device=dev, generator=g0).to(torch.bfloat16)
    w = (torch.randn(Cm, 1, K, device=dev, generator=g0) * 0.5).to(torch.bfloat16)
    b = (torch.randn(Cm, device=dev, generator=g0) * 0.1).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, k=50):
        for _ in range(5):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        barrier()
        return 1e3 * max_over_ranks(e0.elapsed_time(e1)) / k

    def graphed(fn):  # device time only: the call replayed from a CUDA graph
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    g_fused = graphed(lambda: nk.ssd_conv_silu(u, w, b))
    g_torch = graphed(lambda: F.silu(F.conv1d(u.transpose(1, 2), w, b, padding=K - 1, groups=Cm)[..., :Tm]
                                     .transpose(1, 2)).contiguous())
    fused_us = timed(g_fused.replay)
    torch_us = timed(g_torch.replay)
    return {"workload": "silu(causal depthwise conv K=3), B=8, T=2048, C=832 bf16", "fused_us": fused_us,
            "fused_hbm_gbs": Bm * Tm * Cm * 4 / (fused_us / 1e6) / 1e9, "torch_ops_us": torch_us}


def run_assoc(dev, nk, barrier, max_over_ranks):
    """HierarchicalMemory's associative memory at NEED's 350M shape (B=8, T=2048,
    d_model=832, memory_rank=64; fp32 q/k projections, bf16 values): the two
    kernels of linear_associative_memory against the reference's chunked
    computation (need_core.py:1960-2001, chunks of 32) as torch ops on the GPU,
    both replayed from CUDA graphs."""
    import torch
    import torch.nn.functional as F
    g0 = torch.Generator(device=dev).manual_seed(17)
    Bm, Tm, d, r = 8, 2048, 832, 64
    q = torch.randn(Bm, Tm, r, device=dev, generator=g0)
    k = torch.randn(Bm, Tm, r, device=dev, generator=g0)
    v = torch.randn(Bm, Tm, d, device=dev, generator=g0).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def chunked(chunk=32):  # the reference's algorithm, torch ops in the model dtype
        qf = (F.elu(q.float()) + 1.0).to(v.dtype)
        kf = (F.elu(k.float()) + 1.0).to(v.dtype)
        state = v.new_zeros(Bm, r, d)
        den_state = v.new_zeros(Bm, r)
        outs = []
        for s0 in range(0, Tm, chunk):
            qc, kc, vc = qf[:, s0:s0 + chunk], kf[:, s0:s0 + chunk], v[:, s0:s0 + chunk]
            st = state.unsqueeze(1) + (kc.unsqueeze(-1) * vc.unsqueeze(-2)).cumsum(dim=1)
            dn = den_state.unsqueeze(1) + kc.cumsum(dim=1)
            num = torch.einsum("bqr,bqrd->bqd", qc, st)
            outs.append(num / (qc * dn).sum(dim=-1, keepdim=True).clamp_min(1e-6))
            state, den_state = st[:, -1], dn[:, -1]
        return torch.cat(outs, dim=1)

    def graphed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    def timed(graph, k):
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(k):
            graph.replay()
        e1.record(stream)
        barrier()
        return 1e3 * max_over_ranks(e0.elapsed_time(e1)) / k

    kern_us = timed(graphed(lambda: nk.linear_associative_memory(q, k, v)), 30)
    torch_us = timed(graphed(chunked), 3)
    # decode: one token for each of 256 sequences against their states (r x d, bf16)
    Ns = 256
    st = torch.zeros(Ns, r, d, device=dev, dtype=torch.bfloat16)
    dn = torch.zeros(Ns, r, device=dev, dtype=torch.bfloat16)
    qs, ks = torch.randn(Ns, r, device=dev, generator=g0), torch.randn(Ns, r, device=dev, generator=g0)
    vs = torch.randn(Ns, d, device=dev, generator=g0).to(torch.bfloat16)
    step_us = timed(graphed(lambda: nk.assoc_memory_step(qs, ks, vs, st, dn)), 100)
    step_bytes = Ns * (2 * r * d * 2 + 2 * r * 2 + 2 * d * 2 + 2 * r * 4)  # state, denom r/w; v, out; q, k
    # one long sequence: its segments start from chunk states summed once
    Tl = 16384
    ql, kl = torch.randn(1, Tl, r, device=dev, generator=g0), torch.randn(1, Tl, r, device=dev, generator=g0)
    vl = torch.randn(1, Tl, d, device=dev, generator=g0).to(torch.bfloat16)
    long_us = timed(graphed(lambda: nk.linear_associative_memory(ql, kl, vl)), 30)
    long_bytes = 2 * Tl * r * 4 + 2 * Tl * d * 2
    nbytes = 2 * Bm * Tm * r * 4 + 2 * Bm * Tm * d * 2  # q, k (fp32) and v in, out
    tiles = Bm * -(-Tm // 128) * -(-d // 128)
    flops = tiles * 2 * 128 * (128 * 64 + 128 * 128 + 64 * 128 + 128 * 64)  # QK^T, PV, QS, V^T K per tile
    return {"workload": "linear associative memory, B=8, T=2048, d=832, r=64, bf16 values",
            "kernels_us": kern_us, "hbm_gbs": nbytes / (kern_us / 1e6) / 1e9,
            "tensor_tflops": flops / (kern_us / 1e6) / 1e12, "torch_ops_us": torch_us,
            "decode_step": {"workload": "one token for 256 sequences, state 64 x 832 bf16 each",
                            "us": step_us, "hbm_gbs": step_bytes / (step_us / 1e6) / 1e9},
            "long_sequence": {"workload": "one sequence, T=16384, d=832, r=64", "kernels_us": long_us,
                              "hbm_gbs": long_bytes / (long_us / 1e6) / 1e9}}


def run_ssd_block(dev, nk, barrier, max_over_ranks):
    """One StructuredDualRetention forward at NEED's 350M shape (B=8, T=2048,
    d_model=832, conv K=3, dt in [0.001, 0.2], bf16, random weights):
    in-projection, the conv + SiLU prologue, the SSD scan reading the
    projection's chunks in place, RMSNorm and the out-projection
    (need_core.py:1617-1643).  Reports the block's time and the share of the
    two kernels of this repository, and the same with the out_norm as this
    repository's kernel (ssd_scan_rms_norm), all replayed from CUDA graphs."""
    import torch
    import torch.nn.functional as F
    g0 = torch.Generator(device=dev).manual_seed(13)
    Bm, Tm, d = 8, 2048, 832
    bf = torch.bfloat16

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g0) * scale).to(bf)

    x = rnd(Bm, Tm, d)
    w_in, w_out = rnd(5 * d, d, scale=d ** -0.5), rnd(d, d, scale=d ** -0.5)
    conv_w, conv_b = rnd(d, 1, 3, scale=0.5), rnd(d, scale=0.1)
    d_skip = torch.full((d,), 0.1, device=dev)
    norm_w = torch.ones(d, device=dev, dtype=bf)
    proj = F.linear(x, w_in)

    def kernels(p):
        u, bg, cg, dt, og = p.chunk(5, dim=-1)
        return nk.ssd_scan(nk.ssd_conv_silu(u, conv_w, conv_b), bg, cg, dt, og, d_skip, 0.001, 0.2)

    def block():
        return F.linear(F.rms_norm(kernels(F.linear(x, w_in)), (d,), norm_w, 1e-6), w_out)

    def scan_norm(p):  # prologue, then the scan and the out_norm kernel in one call
        u, bg, cg, dt, og = p.chunk(5, dim=-1)
        return nk.ssd_scan_rms_norm(nk.ssd_conv_silu(u, conv_w, conv_b), bg, cg, dt, og, d_skip, 0.001, 0.2,
                                    norm_w, 1e-6)

    def block_fused():
        return F.linear(scan_norm(F.linear(x, w_in)), w_out)

    def folded(p, norm=True):  # the conv folded into the scan's tile loads, then the out_norm kernel
        u, bg, cg, dt, og = p.chunk(5, dim=-1)
        return nk.ssd_conv_scan(u, bg, cg, dt, og, d_skip, 0.001, 0.2, conv_w, conv_b,
                                norm_weight=norm_w if norm else None, eps=1e-6)

    def block_folded():
        return F.linear(folded(F.linear(x, w_in)), w_out)

    stream = torch.cuda.current_stream(dev)

    def graphed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    def timed(graph, k=30):
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(k):
            graph.replay()
        e1.record(stream)
        barrier()
        return 1e3 * max_over_ranks(e0.elapsed_time(e1)) / k

    block_us = timed(graphed(block))
    kernels_us = timed(graphed(lambda: kernels(proj)))
    torch_norm_us = timed(graphed(lambda: F.rms_norm(kernels(proj), (d,), norm_w, 1e-6)))
    need_block_us = timed(graphed(block_fused))
    need_norm_us = timed(graphed(lambda: scan_norm(proj)))
    fold_us = timed(graphed(lambda: folded(proj, norm=False)))
    fold_norm_us = timed(graphed(lambda: folded(proj)))
    fold_block_us = timed(graphed(block_folded))
    return {"workload": "StructuredDualRetention forward, B=8, T=2048, d_model=832, bf16, random weights",
            "block_us": block_us, "prologue_and_scan_us": kernels_us, "scan_share": kernels_us / block_us,
            "block_tokens_per_s": Bm * Tm / (block_us / 1e6),
            "out_norm": {"prologue_scan_then_torch_rms_norm_us": torch_norm_us,
                         "prologue_then_scan_and_rms_norm_kernel_us": need_norm_us,
                         "block_with_rms_norm_kernel_us": need_block_us},
            "conv_folded": {"conv_scan_us": fold_us, "conv_scan_rms_norm_us": fold_norm_us,
                            "block_us": fold_block_us, "block_tokens_per_s": Bm * Tm / (fold_block_us / 1e6)}}


def run_decode(dev, nk, workloads, barrier, max_over_ranks):
    """256 sequences x 4 drafted tokens, verify + commit replayed as one CUDA graph."""
    import torch
    w = workloads.verify(dev, N=256, C=1024, k=4, seed=11)
    pool = w.states.clone()
    y = torch.empty_like(w.x)
    sk = torch.empty_like(w.x)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        nk.ragged_verify(pool, w.cu_k, (w.z, w.g, w.x), out=(y, sk))
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        nk.ragged_verify(pool, w.cu_k, (w.z, w.g, w.x), out=(y, sk))
        nk.commit_states(pool, sk, w.cu_k, w.accept)
    for _ in range(10):
        graph.replay()
    KD = 200
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(KD):
        graph.replay()
    e1.record(stream)
    barrier()
    us = 1e3 * max_over_ranks(e0.elapsed_time(e1)) / KD
    byts = 256 * 1024 * 2 * (1 + 4 * 3 + 4 * 2 + 2)  # state, 3 inputs, y + state per token, commit r/w
    return {"workload": "256 sequences x k=4 drafted tokens, C=1024 bf16 states; verify + commit in one CUDA graph",
            "us_per_step": us, "verified_tokens_per_s": 1024 / (us / 1e6),
            "hbm_gbs": byts / (us / 1e6) / 1e9}


if __name__ == "__main__":
    main()
