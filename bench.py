#!/usr/bin/env python
"""Benchmark of the TRBA INT8-QAT training step on B200.

Metric: QAT train lines/s at 32x160 (TRBA-small: feat_dim 128, 2-layer BiLSTM
hidden 64, max_len 20, 130 classes), one full forward + backward + clip +
Muon/Adam + re-quantisation step per iteration, synthetic data.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B]
    python bench.py --impl reference ...      # the reference's CPU path

One process per GPU (torchrun for N > 1): each rank trains on its own batch
of B lines (weak scaling) and the fp32 gradients are averaged with one NCCL
all-reduce per step before the optimiser.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
METRIC = "QAT train lines/s (TRBA 32x160)"


def load_package():
    name = "trba_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = REPO / "trba-rust_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=512, help="lines per GPU per step")
    ap.add_argument("--img-w", type=int, default=160)
    ap.add_argument("--max-len", type=int, default=20)
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm-sweep", action="store_true")
    ap.add_argument("--aux-out", default=None, help="also write the auxiliary JSON lines to this file")
    ap.add_argument("--eager", action="store_true", help="launch the step kernel by kernel (no CUDA graph)")
    ap.add_argument("--dgrad-mode", type=int, default=1, choices=[0, 1],
                    help="conv input gradient: 0 exact f32 order (CUDA cores), 1 tensor cores")
    ap.add_argument("--mope", action="store_true",
                    help="MoPE inference serving: 9 length-bucket experts, greedy decoding (not the training metric)")
    ap.add_argument("--mope-lines", type=int, default=65536)
    ap.add_argument("--preproc", action="store_true",
                    help="line-image preprocessing (load_image_q) throughput instead of the training step")
    ap.add_argument("--preproc-lines", type=int, default=512)
    ap.add_argument("--mope-batch", type=int, default=512)
    ap.add_argument("--gemm-shape", default=None,
                    help="M,N,K: time only the int8 GEMM (s32 and fused int8 epilogue) at this shape")
    ap.add_argument("--dgrad-shape", default=None,
                    help="B,Cin,H,W,Cout,kh,kw,sh,sw,ph,pw: time only the tensor-core conv input gradient "
                         "(trba_conv_grad_input_i8_tc) at this shape")
    ap.add_argument("--conv-shape", default=None,
                    help="B,Cin,H,W,Cout,kh,kw,sh,sw,ph,pw: time only the implicit-GEMM conv forward "
                         "(trba_conv_gemm_int8_implicit) against im2col + GEMM at this shape")
    ap.add_argument("--dgrad-tiling", default="0,0",
                    help="mb,kc of the tensor-core input gradient (trba_tc_dgrad_tiling): -1,0 class tiling "
                         "for every conv, 0,0 automatic, else a forced halo tile")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0)))


# ----------------------------------------------------------------- clocks --
class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev, self.p = dev, None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-i", str(self.dev), "-lms", "200"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if not self.p:
            return None
        time.sleep(0.25)
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 6:
                continue
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[2:6]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def metric_name(args) -> str:
    return METRIC if args.img_w == 160 else f"QAT train lines/s (TRBA 32x{args.img_w})"


def workload_config(args, world: int) -> dict:
    """The `config` object both arms print: the workload, never the sample."""
    return {"workload": f"TRBA-small QAT train step 32x{args.img_w}, max_len {args.max_len}, "
                        f"batch {args.batch} per GPU",
            "img": f"3x32x{args.img_w}", "feat_dim": 128, "hidden": 64, "classes": 130,
            "max_len": args.max_len, "global_batch": args.batch * world, "per_gpu_batch": args.batch,
            "parallelism": f"dp{world}", "l2": "working set > 126 MB L2 (activations of a step)"}


# Lines per step of the CPU samples: the reference's own CPU path takes about
# 30 ms per 32x160 line on 16 host cores, so 48 lines (the reference's
# training batch) keep each sampled step near 1.5 s.
CPU_SAMPLE_LINES = 48


# ------------------------------------------------------------ reference --
def cpu_step_sample(lines: int, steps: int, warmup: int, img_w: int, max_len: int, seed: int):
    """Times the reference's CPU path (oracle/step_oracle.py driving the
    reference's own CPU backend, oracle/_ref, OpenMP on every host core) on
    `lines` lines per step; returns (lines/s, cores, backend name)."""
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    sys.path.insert(0, str(REPO / "oracle"))
    import step_oracle as so
    ref = REPO / "oracle" / "_ref" / "libtrba_ref_omp.so"
    be = so.CpuBackend(ref if ref.exists() else REPO / "oracle" / "liboracle.so")
    cfg = so.Config(img_w=img_w, max_len=max_len)
    orc = so.OracleTrba(cfg, so.init_params(cfg, seed), be)
    batches = [so.make_batch(cfg, lines, seed + i) for i in range(2)]
    for i in range(warmup):
        orc.train_step(*batches[i % 2])
    t0 = time.perf_counter()
    for i in range(steps):
        orc.train_step(*batches[i % 2])
    dt = time.perf_counter() - t0
    kind = "reference" if be.path.name == "libtrba_ref_omp.so" else "port"
    return lines * steps / dt, cores, kind, be.path.name


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # Bounded sample of the same workload: every step trains CPU_SAMPLE_LINES
    # lines of it (the full per-GPU batch would take minutes per step on the
    # host); lines/s is the same metric.
    lines = CPU_SAMPLE_LINES
    v, cores, kind, lib = cpu_step_sample(lines, args.steps, args.warmup, args.img_w, args.max_len, args.seed)
    sample = (f"{lines} lines of the workload per step x {args.steps} timed steps (after {args.warmup} warm-up), "
              f"{lib}, OMP {cores} threads")
    print(json.dumps({
        "impl": "reference", "metric": metric_name(args), "value": v, "unit": "lines/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * lines / v, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (s8xs8->s32) / fp32", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": v, "unit": "lines/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": v, "unit": "lines/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------------ ours --
def measured_peaks() -> dict:
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def int8_gemm_peak(dev) -> float:
    """cuBLAS int8 GEMM throughput (TOP/s) at 8192^3 on this GPU: the
    measured denominator of the int8 tensor-core roofline."""
    import torch
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(10):
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    torch.cuda.empty_cache()
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


GEMM_SWEEP = [(m, n, k) for m in (6144, 24576, 98304) for n in (64, 128, 256, 512) for k in (64, 576, 1152, 2304)]


def gemm_sweep(L, dev, int8_peak: float, hbm_gbs: float | None, reps: int = 5) -> dict:
    """The standalone int8 GEMM sweep (48 im2col / gate GEMM shapes): every
    shape through launch_gemm_int8 (s32 out) and trba_gemm_int8_requant
    (fused int8 out), each launch timed alone with CUDA events after an L2
    flush (a 256 MB memset), best of `reps`.  Reported per shape: TOP/s,
    fraction of the cuBLAS int8 peak and of max(ops/peak, bytes/HBM) — the
    roofline time of that shape's algorithmic bytes."""
    import torch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g = torch.Generator(device=dev).manual_seed(3)
    rows = []
    mmax, nmax, kmax = 98304, 512, 2304
    A = torch.randint(-127, 128, (mmax, kmax), dtype=torch.int8, device=dev, generator=g)
    B = torch.randint(-127, 128, (nmax, kmax), dtype=torch.int8, device=dev, generator=g)
    C32 = torch.empty(mmax * nmax, dtype=torch.int32, device=dev)
    C8 = torch.empty(mmax * nmax, dtype=torch.int8, device=dev)
    bias = torch.zeros(nmax, dtype=torch.float32, device=dev)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    for (m, n, k) in GEMM_SWEEP:
        a = A[:m, :k].contiguous()
        b = B[:n, :k].contiguous()
        res = {}
        for name in ("s32", "requant_i8"):
            best = float("inf")
            for _ in range(reps + 1):
                flush.zero_()
                e0.record()
                if name == "s32":
                    L.launch_gemm_int8(p(a), p(b), p(C32), m, n, k, None)
                else:
                    L.trba_gemm_int8_requant(p(a), p(b), p(bias), p(C8), m, n, k, 127.0 * 64.0, 50.0, None)
                e1.record()
                e1.synchronize()
                best = min(best, e0.elapsed_time(e1))
            ops = 2.0 * m * n * k
            nbytes = m * k + n * k + (4 if name == "s32" else 1) * m * n
            t_roof = max(ops / (int8_peak * 1e12), nbytes / (hbm_gbs * 1e9)) if hbm_gbs else ops / (int8_peak * 1e12)
            res[name] = {"us": best * 1e3, "tops": ops / (best * 1e-3) / 1e12,
                         "frac_peak": ops / (best * 1e-3) / 1e12 / int8_peak,
                         "frac_roofline": t_roof / (best * 1e-3),
                         "compute_bound": ops / (int8_peak * 1e12) >= (nbytes / (hbm_gbs * 1e9) if hbm_gbs else 0)}
        rows.append({"m": m, "n": n, "k": k, **res})
    del A, B, C32, C8, flush
    torch.cuda.empty_cache()
    if L.trba_tc_error_poll(1) != 0:
        raise RuntimeError("tensor-core GEMM reported a timed-out wait during the sweep")
    cb = [r for r in rows if r["requant_i8"]["compute_bound"]]
    return {
        "shapes": len(rows), "peak_tops": int8_peak, "unit": "TOP/s",
        "best_tops_s32": max(r["s32"]["tops"] for r in rows),
        "best_tops_requant_i8": max(r["requant_i8"]["tops"] for r in rows),
        "compute_bound_requant_i8": [{"shape": [r["m"], r["n"], r["k"]], "tops": r["requant_i8"]["tops"],
                                      "frac_peak": r["requant_i8"]["frac_peak"]} for r in cb],
        "median_frac_roofline_s32": statistics.median(r["s32"]["frac_roofline"] for r in rows),
        "median_frac_roofline_requant_i8": statistics.median(r["requant_i8"]["frac_roofline"] for r in rows),
        "per_shape": rows,
    }


def profiled_traffic(kernel: str, batch: int):
    """DRAM bytes per launch of `kernel` at this batch, from the committed ncu
    summary profiles/<kernel>_traffic.txt (line 'bytes_per_launch_per_line:
    X', DRAM read + write per launch divided by the batch the capture ran
    at; traffic grows with the batch).  None when no capture is committed."""
    f = REPO / "profiles" / f"{kernel}_traffic.txt"
    try:
        for line in f.read_text().splitlines():
            if line.startswith("bytes_per_launch_per_line:"):
                return float(line.split(":", 1)[1]) * batch
    except OSError:
        pass
    return None



def our_arm(args):
    import numpy as np
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    pkg = load_package()
    from trba_b200 import data, dp
    from trba_b200.model import Config, QatModel
    L = pkg.lib()
    L.trba_tc_dgrad_tiling(*(int(x) for x in args.dgrad_tiling.split(",")))
    cfg = Config(img_w=args.img_w, max_len=args.max_len, batch=args.batch, dgrad_mode=args.dgrad_mode)
    m = QatModel(cfg)
    m.set_params(data.init_params(m.manifest(), cfg, args.seed))
    if world > 1:
        dp.join(m)
    host = data.make_batch(cfg, args.batch, dp.rank_seed(args.seed, rank))
    pinned = [torch.from_numpy(a).pin_memory() for a in host]
    devb = [p.to(dev) for p in pinned]
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    # measured ceilings for the roofline, taken before the timed region
    f32_peak = C.c_double()
    if L.trba_measure_f32_muladd_peak(C.byref(f32_peak), sptr) != 0:
        raise RuntimeError(L.trba_last_error_string().decode())
    int8_peak = int8_gemm_peak(dev) if rank == 0 else None

    # The dominant kernel (the conv input-gradient gather) is timed on the
    # stream it runs on.  Eager steps (--eager): CUDA events around every
    # launch of the timed region.  Graph replays (default): the probe is
    # recorded into the step graph (set before the warm-up, which records the
    # graph); each launch is bracketed by device %globaltimer stamps (events
    # recorded inside a graph cannot be timed), read for the last timed step.
    graphs = not args.eager
    m.use_graphs(graphs)
    if graphs:
        m.probe(m.PROBE_DGRAD)
    for _ in range(max(3, args.warmup)):
        m.train_step(*devb, stream=sptr)
    barrier()
    clocks = Clocks(local)
    clocks.start()
    l0 = L.trba_launch_count()
    if not graphs:
        m.probe(m.PROBE_DGRAD)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        m.train_step(*devb, stream=sptr)
    e1.record(stream)
    # NCCL failure detection: a rank whose peer failed (or never joined) aborts
    # its communicator instead of hanging in the next synchronisation
    if world > 1 and m.dp_wait(sptr, timeout_s=120.0) != 0:
        raise RuntimeError("data-parallel step failed: the NCCL communicator was aborted")
    barrier()
    ck = clocks.stop()
    launches = (L.trba_launch_count() - l0) / args.steps
    dg_ms, dg_n, dg_ops, dg_bytes, dg_steps = m.probe_read()
    ms = dp.max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    loss = m.loss()
    value = args.batch * world / (ms / 1000.0)

    # end to end through the host-buffer entry point: H2D inputs + D2H loss in every step
    e2e = None
    if not args.no_e2e:
        np_in = [p.numpy() for p in pinned]
        m.train_step_host(*np_in, stream=sptr)
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            m.train_step_host(*np_in, stream=sptr)
        e1.record(stream)
        barrier()
        ms2 = dp.max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
        h2d = sum(int(a.nbytes) for a in np_in)
        e2e = {"value": args.batch * world / (ms2 / 1000.0), "unit": "lines/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 12}

    m.probe(-1)
    # int8 tensor-core GEMMs of the step (forward conv + weight gradient),
    # probed over a few eager steps after the timed region
    m.use_graphs(False)
    gemm = {}
    for name, kind in (("conv_fwd", m.PROBE_CONV_GEMM), ("conv_wgrad", m.PROBE_WGRAD_GEMM),
                       ("head_sgemm_f64acc", m.PROBE_SGEMM)):
        m.probe(kind)
        for _ in range(3):
            m.train_step(*devb, stream=sptr)
        g_ms, g_n, g_ops, g_bytes, _ = m.probe_read()
        m.probe(-1)
        gemm[name] = {"launches_per_step": g_n // 3, "ms_per_step": g_ms / 3,
                      "tops": g_ops / (g_ms * 1e-3) / 1e12 if g_ms > 0 else None}
    # where the step's time goes: each phase spanned on the step's stream
    phases = {}
    for name, kind in m.PROBE_PHASES.items():
        m.probe(kind)
        for _ in range(3):
            m.train_step(*devb, stream=sptr)
        p_ms, _, _, _, _ = m.probe_read()
        m.probe(-1)
        phases[name] = p_ms / 3
    barrier()

    sweep = None
    if rank == 0 and world == 1 and not args.no_gemm_sweep and int8_peak:
        sweep = gemm_sweep(L, dev, int8_peak, measured_peaks().get("hbm_gbs"))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        lines, steps = CPU_SAMPLE_LINES, 8
        v, cores, kind, lib = cpu_step_sample(lines, steps, 1, args.img_w, args.max_len, args.seed)
        cpu = {"value": v, "unit": "lines/s", "cores": cores, "kind": kind,
               "sample": f"{lines} lines of the workload per step x {steps} timed steps (1 warm-up), {lib}, "
                         f"OMP {cores} threads"}

    roofline = None
    if dg_n > 0 and dg_ms > 0:
        per_launch_s = dg_ms * 1e-3 / dg_n
        useful = dg_ops / dg_n / per_launch_s / 1e12  # fp32-equivalent multiply-adds of the gather terms
        hbm = measured_peaks().get("hbm_gbs")
        if args.dgrad_mode == 1:
            # tensor cores: dy enters as three bf16 terms, so the MMA work of
            # the exact product is three times the useful multiply-adds
            peak = measured_peaks().get("bf16_tflops_sustained")
            achieved = 3.0 * useful
            traffic = profiled_traffic("dgrad_halo_kernel", args.batch)
            roofline = {
                "kernel": "dgrad_halo_kernel + split_halo_kernel: conv input gradient, implicit GEMM on tcgen05 "
                          "(kind::f16, dy as three exact bf16 terms, one shared-memory halo per tile)",
                "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak if peak else None,
                "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained (the kernel runs inside a long step)",
                "useful_fp32_equiv_tflops": useful,
            }
        else:
            traffic = profiled_traffic("dgrad_kernel", args.batch)
            roofline = {
                "kernel": "dgrad_kernel: conv input gradient, f32 in the reference's summation order",
                "bound": "fp32", "achieved": useful, "peak": f32_peak.value, "unit": "TFLOP/s",
                "frac": useful / f32_peak.value,
                "peak_source": "measured in this run: separately rounded f32x2 multiply + add chains on every SM",
            }
        roofline.update({
            "traffic": traffic,
            "algorithmic_bytes_per_launch": dg_bytes / dg_n,
            "hbm_gbs_at_algorithmic_bytes": dg_bytes / dg_n / per_launch_s / 1e9,
            "hbm_peak_gbs": hbm,
            "launches_per_step": dg_n / dg_steps,
            "ms_per_step": dg_ms / dg_steps,
            "share_of_step": dg_ms / dg_steps / ms,
        })
    gemm_line = None
    head = gemm.pop("head_sgemm_f64acc")
    if int8_peak:
        tot_ms = sum(g["ms_per_step"] for g in gemm.values())
        tot_tops = sum((g["tops"] or 0) * g["ms_per_step"] for g in gemm.values()) / tot_ms if tot_ms else None
        gemm_line = {"bound": "tensor", "achieved": tot_tops, "peak": int8_peak, "unit": "TOP/s",
                     "frac": tot_tops / int8_peak if tot_tops else None,
                     "peak_source": "measured in this run: torch._int_mm (cuBLAS) int8 8192^3, best of 10",
                     "by_gemm": gemm}
    if rank == 0:
        # Auxiliary lines first (one JSON object per line, each tagged "aux"),
        # the headline last and short: the driver parses the final line.
        aux = []
        if sweep:
            for r in sweep.pop("per_shape"):
                aux.append({"aux": "int8_gemm_sweep_shape", **r})
            aux.append({"aux": "int8_gemm_sweep_summary", **sweep})
        if gemm_line:
            aux.append({"aux": "roofline_int8_gemm", **gemm_line})
        aux.append({"aux": "head_sgemm", "launches_per_step": head["launches_per_step"],
                    "ms_per_step": head["ms_per_step"], "tflops": head["tops"]})
        aux.append({"aux": "step_phases_ms", **phases,
                    "note": "eager steps, each phase spanned on the step's stream"})
        aux.append({"aux": "loss_last", "loss": [float(x) for x in loss]})
        for a in aux:
            print(json.dumps(a), flush=True)
        if args.aux_out:
            Path(args.aux_out).parent.mkdir(parents=True, exist_ok=True)
            Path(args.aux_out).write_text("\n".join(json.dumps(a) for a in aux) + "\n")
        summary = None
        if sweep:
            summary = {"peak_tops": sweep["peak_tops"],
                       "best_frac_requant_i8_compute_bound": max(
                           (c["frac_peak"] for c in sweep["compute_bound_requant_i8"]), default=None)}
        out = {
            "metric": metric_name(args), "value": value, "unit": "lines/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 (s8xs8->s32) / fp32", "data": "synthetic",
            "config": workload_config(args, world),
            "gpu_launches": launches,
            "clocks": ck,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "roofline": roofline,
            "int8_gemm": summary,
        }
        line = json.dumps(out)
        if len(line) > 4000:  # keep the headline short whatever the optional parts hold
            out.pop("int8_gemm")
            out["roofline"] = {k: roofline[k] for k in ("bound", "achieved", "peak", "unit", "frac", "traffic")}
            line = json.dumps(out)
        print(line, flush=True)
    m.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def gemm_only(args):
    """One GEMM shape, s32 and fused-int8 outputs (for profiling one launch)."""
    import torch
    m, n, k = (int(x) for x in args.gemm_shape.split(","))
    pkg = load_package()
    L = pkg.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    kp = (k + 15) & ~15
    a = torch.randint(-127, 128, (m, kp), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (n, kp), dtype=torch.int8, device=dev, generator=g)
    c32 = torch.empty((m, n), dtype=torch.int32, device=dev)
    c8 = torch.empty((m, n), dtype=torch.int8, device=dev)
    bias = torch.zeros(n, dtype=torch.float32, device=dev)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    out = {"gemm": [m, n, k]}
    for name in ("s32", "requant_i8"):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(max(3, args.steps)):
            e0.record()
            if name == "s32":
                L.launch_gemm_int8(p(a), p(b), p(c32), m, n, k, None)
            else:
                L.trba_gemm_int8_requant(p(a), p(b), p(bias), p(c8), m, n, k, 127.0 * 64.0, 50.0, None)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        out[name] = {"us": best * 1e3, "tops": 2.0 * m * n * k / (best * 1e-3) / 1e12}
    # the same s32 GEMM on one CTA per tile (pair kernel off) and through cuBLAS, for context
    prev = L.trba_gemm_pair_enable(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(max(3, args.steps)):
        e0.record()
        L.launch_gemm_int8(p(a), p(b), p(c32), m, n, k, None)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    L.trba_gemm_pair_enable(prev)
    out["s32_single_cta"] = {"us": best * 1e3, "tops": 2.0 * m * n * k / (best * 1e-3) / 1e12}
    try:
        bt = b[:, :k].t()
        a_k = a[:, :k].contiguous()
        best = float("inf")
        for _ in range(max(3, args.steps)):
            e0.record()
            torch._int_mm(a_k, bt)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        out["cublas_s32"] = {"us": best * 1e3, "tops": 2.0 * m * n * k / (best * 1e-3) / 1e12}
    except Exception as exc:  # pragma: no cover - shape constraints of the library call
        out["cublas_s32"] = {"unavailable": str(exc)[:120]}
    if L.trba_tc_error_poll(1) != 0:
        raise RuntimeError("tensor-core GEMM reported a timed-out wait")
    print(json.dumps(out), flush=True)


def dgrad_only(args):
    """One conv input-gradient shape through trba_conv_grad_input_i8_tc (for
    timing and profiling one kernel): per-call device time with CUDA events
    (weight image, dy split and the tensor-core GEMM), after 3 warm-up calls."""
    import torch
    B, cin, h, w, cout, kh, kw, sh, sw, ph, pw = (int(x) for x in args.dgrad_shape.split(","))
    ho, wo = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
    pkg = load_package()
    L = pkg.lib()
    L.trba_tc_dgrad_tiling(*(int(x) for x in args.dgrad_tiling.split(",")))
    plan = (C.c_longlong * 80)()
    nf = L.trba_tc_dgrad_plan(B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo, plan, 80)
    names = "halo BN Npad ntn tiles ntaps KC nchunks mb R sa sb Hq Wq dmin mpos rows".split()
    plan_info = dict(zip(names, list(plan[:min(nf, len(names))])))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    kp = (cin * kh * kw + 15) & ~15
    dy = torch.randn((B, cout, ho, wo), device=dev, generator=g) * 1e-3
    wq = torch.randint(-127, 128, ((cout + 15) & ~15, kp), dtype=torch.int8, device=dev, generator=g)
    gi = torch.empty((B, cin, h, w), device=dev)
    a = (C.c_void_p(dy.data_ptr()), C.c_void_p(wq.data_ptr()), kp, 0.01, C.c_void_p(gi.data_ptr()), B, cin, h, w,
         cout, kh, kw, sh, sw, ph, pw, ho, wo, None)
    for _ in range(3):
        if L.trba_conv_grad_input_i8_tc(*a) != 0:
            raise RuntimeError(L.trba_last_error_string().decode())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(1, args.steps)
    e0.record()
    for _ in range(n):
        L.trba_conv_grad_input_i8_tc(*a)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n
    vy = sum(1 for y in range(h) for t in range(kh) if (y + ph - t) >= 0 and (y + ph - t) % sh == 0 and (y + ph - t) // sh < ho)
    vx = sum(1 for x in range(w) for t in range(kw) if (x + pw - t) >= 0 and (x + pw - t) % sw == 0 and (x + pw - t) // sw < wo)
    flops = 2.0 * B * cin * cout * vy * vx
    if L.trba_tc_error_poll(1) != 0 or L.trba_last_error() != 0:
        raise RuntimeError("input-gradient kernel reported an error")
    print(json.dumps({"dgrad": [B, cin, h, w, cout, kh, kw, sh, sw, ph, pw], "plan": plan_info, "us_per_call": us,
                      "useful_tflops": flops / (us * 1e-6) / 1e12,
                      "bf16_mma_tflops_three_terms": 3 * flops / (us * 1e-6) / 1e12}), flush=True)


def conv_only(args):
    """One conv forward shape: im2col + GEMM (launch_im2col_pad,
    launch_gemm_int8) against the implicit GEMM (trba_conv_gemm_int8_implicit:
    NHWC copy of the input, weight re-order, gathered-operand GEMM), per-call
    device time with CUDA events after 3 warm-up calls, s32 results compared."""
    import torch
    B, cin, h, w, cout, kh, kw, sh, sw, ph, pw = (int(x) for x in args.conv_shape.split(","))
    ho, wo = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
    L = load_package().lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    k = cin * kh * kw
    kp, rows = (k + 15) & ~15, B * ho * wo
    x = torch.randint(-127, 128, (B, cin, h, w), dtype=torch.int8, device=dev, generator=g)
    wq = torch.randint(-127, 128, ((cout + 15) & ~15, kp), dtype=torch.int8, device=dev, generator=g)
    col = torch.zeros(((rows + 15) & ~15, kp), dtype=torch.int8, device=dev)
    acc0 = torch.empty((rows, cout), dtype=torch.int32, device=dev)
    acc1 = torch.empty((rows, cout), dtype=torch.int32, device=dev)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def two_launch():
        L.launch_im2col_pad(p(x), p(col), B, cin, h, w, kh, kw, sh, sw, ph, pw, ho, wo, kp, None)
        L.launch_gemm_int8(p(col), p(wq), p(acc0), rows, cout, k, None)

    def implicit():
        if L.trba_conv_gemm_int8_implicit(p(x), p(wq), kp, p(acc1), B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho,
                                          wo, None) != 0:
            raise RuntimeError(L.trba_last_error_string().decode())

    out = {"conv": [B, cin, h, w, cout, kh, kw, sh, sw, ph, pw]}
    n = max(1, args.steps)
    for name, fn in (("im2col_gemm_us", two_launch), ("implicit_us", implicit)):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        e1.synchronize()
        out[name] = e0.elapsed_time(e1) * 1e3 / n
    if not torch.equal(acc0, acc1):
        raise RuntimeError("implicit conv GEMM differs from im2col + GEMM")
    if L.trba_tc_error_poll(1) != 0 or L.trba_last_error() != 0:
        raise RuntimeError("conv kernels reported an error")
    ops = 2.0 * rows * cout * k
    out["implicit_tops"] = ops / (out["implicit_us"] * 1e-6) / 1e12
    # algorithmic bytes of the implicit conv: int8 input + weights + s32 output
    out["implicit_gbs_algorithmic"] = (B * cin * h * w + cout * k + 4.0 * rows * cout) / (out["implicit_us"] * 1e-6) / 1e9
    print(json.dumps(out), flush=True)


def mope_arm(args):
    """MoPE inference serving: synthetic lines with the documented length
    histogram, routed to 9 length-bucket experts placed on the ranks by
    expected work; each rank decodes its experts' lines greedily.  value =
    all lines / max over ranks of the device-timed decoding (CUDA events,
    including the per-batch token copy and the output rule)."""
    import numpy as np
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    load_package()
    from trba_b200 import dp, mope
    experts = mope.default_experts()
    lengths = mope.synthetic_lengths(args.mope_lines, args.seed)
    eidx = mope.route(lengths, experts)
    counts = np.bincount(eidx, minlength=len(experts)).tolist()
    plan = mope.place(experts, counts, world)
    mine = [i for i in range(len(experts)) if plan[i] == rank]
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    runners, imgs = {}, {}
    for i in mine:
        e = experts[i]
        runners[i] = mope.ExpertRunner(e, args.mope_batch, args.seed + i)
        # uniform [0, 1] pixels quantised to int8 (scale 1/127)
        imgs[i] = torch.randint(0, 128, (counts[i], 3, 32, e.img_w), dtype=torch.int8, device=dev, generator=g)
    for i in mine:  # warm-up: one decoding batch per expert
        runners[i].decode(imgs[i][:args.mope_batch])
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    out = {}
    for i in mine:
        out[i] = runners[i].decode(imgs[i])
    e1.record()
    torch.cuda.synchronize(dev)
    ms = dp.max_over_ranks(e0.elapsed_time(e1), dev)
    mem = max(int(runners[i].model.L.trba_model_device_bytes(runners[i].model.h)) for i in mine) if mine else 0
    decoded = sum(len(v) for v in out.values())
    total = torch.tensor([decoded], device=dev)
    if world > 1:
        torch.distributed.all_reduce(total)
    if rank == 0:
        print(json.dumps({
            "metric": "MoPE int8 inference lines/s (9 length-bucket experts, greedy decoding)",
            "value": int(total.item()) / (ms / 1000.0), "unit": "lines/s", "n_gpus": world,
            "ms_total": ms, "higher_is_better": True, "scaling": "strong", "data": "synthetic",
            "config": {"workload": f"{args.mope_lines} lines, length histogram p50 5 / p90 11 / max 32",
                       "experts": [[e.name, e.img_w, e.max_len, c, r] for e, c, r in zip(experts, counts, plan)],
                       "batch_per_call": args.mope_batch, "placement": "greedy by expected work",
                       "max_expert_device_bytes": mem},
        }), flush=True)
    for r in runners.values():
        r.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def synthetic_line_images(n: int, seed: int):
    """Decoded RGB8 line images: height 48..160 px, width 4..16x the height,
    light paper with dark strokes (seeded)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        h = int(rng.integers(48, 161))
        w = int(h * rng.uniform(4.0, 16.0))
        im = np.full((h, w, 3), 235, np.uint8)
        strokes = rng.random((h, w)) < 0.08
        im[strokes] = rng.integers(0, 80, (int(strokes.sum()), 1), dtype=np.uint8)
        out.append(im)
    return out


def preproc_arm(args):
    """load_image_q on the device for a batch of decoded line images.  value:
    device-timed lines/s with the pixels resident (CUDA events around the
    kernel, L2 flushed before each step); e2e: the same through
    preprocess_lines' path with the H2D copy of the packed pixels from pinned
    memory inside the timed region (the int8 batch stays on the device for
    the model); cpu_baseline: the CPU restatement (oracle/preproc_oracle.py,
    numpy, one thread) on a sample of the same images."""
    import numpy as np
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    load_package()
    from trba_b200 import preproc as pp
    imgs = synthetic_line_images(args.preproc_lines, args.seed + rank)
    packed = pp.PackedImages(imgs)
    batch = pp.DeviceBatch(packed, dev)
    out = torch.empty((len(imgs), 32 * 160 * 3), dtype=torch.int8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        pp.preprocess_device(batch, 32, 160, out)
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, b in ev:
        flush.zero_()
        a.record()
        pp.preprocess_device(batch, 32, 160, out)
        b.record()
    torch.cuda.synchronize(dev)
    ms = sorted(a.elapsed_time(b) for a, b in ev)[len(ev) // 2]
    e2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, b in e2:
        flush.zero_()
        a.record()
        bt = pp.DeviceBatch(packed, dev)
        pp.preprocess_device(bt, 32, 160, out)
        b.record()
    torch.cuda.synchronize(dev)
    ms_e2e = sorted(a.elapsed_time(b) for a, b in e2)[len(e2) // 2]
    src_px = int(sum(im.shape[0] * im.shape[1] for im in imgs))
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        sys.path.insert(0, str(REPO / "oracle"))
        import preproc_oracle as po
        k = min(len(imgs), 16)
        t0 = time.perf_counter()
        for im in imgs[:k]:
            po.load_image_q(im, 32, 160)
        dt = time.perf_counter() - t0
        cpu = {"value": k / dt, "unit": "lines/s", "cores": 1, "kind": "port",
               "sample": f"{k} of the same images through the numpy restatement"}
    if rank == 0:
        print(json.dumps({
            "metric": "line-image preprocessing lines/s (decoded RGB8 -> 32x160 int8 model input)",
            "value": len(imgs) / (ms / 1000.0), "unit": "lines/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
            "dtype": "u8 -> f32 -> int8", "data": "synthetic",
            "config": {"workload": f"{len(imgs)} line images, height 48..160, width 4..16x height",
                       "source_megapixels": src_px / 1e6, "l2": "256 MB flush before each step"},
            "e2e": {"value": len(imgs) / (ms_e2e / 1000.0), "unit": "lines/s",
                    "h2d_bytes_per_step": packed.nbytes + 16 * len(imgs), "d2h_bytes_per_step": 0},
            "gpu_launches": 1, "cpu_baseline": cpu,
        }), flush=True)


def main():
    args = parse()
    if args.preproc:
        preproc_arm(args)
        return
    if args.mope:
        mope_arm(args)
        return
    if args.gemm_shape:
        gemm_only(args)
        return
    if args.dgrad_shape:
        dgrad_only(args)
        return
    if args.conv_shape:
        conv_only(args)
        return
    if args.impl == "reference":
        reference_arm(args)
    else:
        our_arm(args)


if __name__ == "__main__":
    main()
