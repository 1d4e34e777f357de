#!/usr/bin/env python
"""Benchmark of the quantized-weight decode path: Q4_K GEMV weight GB/s.

Workload: W = 11008 x 4096 in GGUF Q4_K (25,362,432 bytes of blocks), one bf16
activation row (M = 1), fp32 output -- the decode point of the Q4_K
dequant-GEMM sweep.  One step = that activation row through 16 distinct
weight matrices of this shape (16 calls of the fused dequant-GEMV, one kernel
each: a stack of 16 projection layers, 406 MB of blocks, more than 3x the
126 MB L2), so every launch streams its weight from HBM and the timed region
holds 16 launches per step.  Weights and activations are seeded synthetic
data (random-init blocks with the documented value distributions).

Printed line (rank 0): ``value`` = quantized weight bytes of all steps of all
ranks / max-over-ranks device time of the timed graph replay; ``e2e`` = the
same metric through the public ``LinearOp.forward`` with the activation coming
from pinned host memory and the result read back every call; ``roofline`` =
the GEMV kernel against the measured HBM copy bandwidth; ``check`` = the
headline's outputs against the oracle's fp32 ``x @ W.T`` on the reference's
fp16 weights; ``cpu_baseline`` = the numpy restatement of the reference's path
(fp32 x @ W.T on the dequantized weight) on this host's cores.  The same line
carries the other configurations (Q8_0 dequant + GEMV, Q6_K/Q5_K decode
shapes, the prefill GEMM sweep, Llama decode and prefill, the MoE block).

``--impl reference`` times the reference's CPU path (the numpy port in
``oracle/``) on the same workload instead.  Multi-GPU (torchrun): every rank
runs the same per-GPU workload on its own weights (weak scaling; the row
blocks are independent, so there is no collective in the data path); the
Llama decode section is tensor-parallel over all ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

QTYPE, N, K, M = "Q4_K", 11008, 4096, 1
W_BYTES = N * (K // 256) * 144          # 25,362,432
COPIES = 16                             # distinct weights per step
METRIC = "Q4_K GEMV weight GB/s"
UNIT = "GB/s"
# DRAM bytes read+written per launch of the GEMV kernel on this shape, from an
# ncu capture of this bench's GEMV (dram__bytes_read.sum + dram__bytes_write.sum).
NCU_TRAFFIC_PER_LAUNCH = 25_409_536
KERNEL = "k_qgemv_q4k_k4096_m1<bf16> (fused activation split)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the prefill (tensor-core GEMM) sweep")
    ap.add_argument("--no-configs", action="store_true", help="skip the Q8_0 / Q6_K / Q5_K / dequant sections")
    ap.add_argument("--moe", action="store_true",
                    help="only time the Mixtral-shape MoE block (8 experts, top-2, 1024 tokens, 4096 -> 14336)")
    ap.add_argument("--no-decode", action="store_true", help="skip the Llama decode / prefill section")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE block section")
    ap.add_argument("--decode-steps", type=int, default=64)
    ap.add_argument("--decode-profile", type=int, default=0,
                    help="profiling mode: two graph-replayed decode steps of this batch size between "
                         "cudaProfilerStart/Stop (with --decode-layers layers)")
    ap.add_argument("--decode-layers", type=int, default=2)
    ap.add_argument("--prefill-profile", type=int, default=0,
                    help="profiling mode: a prefill of this many tokens (batch 1, --decode-layers layers) "
                         "between cudaProfilerStart/Stop")
    ap.add_argument("--gemm-m", type=int, default=0,
                    help="only time the prefill GEMM with this many activation rows (profiling mode)")
    ap.add_argument("--gemm-type", default="Q4_K", help="block type of --gemm-m / --gemv-only")
    ap.add_argument("--gemm-n", type=int, default=N)
    ap.add_argument("--gemm-k", type=int, default=K)
    ap.add_argument("--gemv-only", type=int, default=0,
                    help="profiling mode: only this many GEMV launches of --gemm-type (--gemm-n x --gemm-k, "
                         "fp32 x of --gemv-m rows)")
    ap.add_argument("--gemv-m", type=int, default=1)
    ap.add_argument("--dequant-only", type=int, default=0,
                    help="profiling mode: only this many dequant launches of --gemm-type (--gemm-n x --gemm-k)")
    return ap.parse_args()


def config():
    """The workload description; identical in both arms."""
    return {"workload": f"{QTYPE} GEMV {N}x{K}, M={M}, bf16 activations, fp32 out; one step = the row through "
                        f"{COPIES} distinct weights of this shape",
            "weight_bytes": W_BYTES, "weights_per_step": COPIES,
            "l2_policy": f"inputs larger than L2: {COPIES} distinct weights = {COPIES * W_BYTES / 1e6:.0f} MB per step",
            "parallelism": "independent replicas per GPU (row blocks), no collective"}


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        self.idx = ids[gpu_index] if gpu_index < len(ids) and ids[gpu_index].isdigit() else gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r.split(",") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's per-step work (fp32 x @ W.T on the weight it
# dequantized at load), restated in numpy in oracle/
# ---------------------------------------------------------------------------
def cpu_port_setup(raw, x_bf16_as_f32):
    from oracle import gguf_dequant_oracle as O
    w32 = O.dequantize(raw, QTYPE, (N, K)).astype(np.float32)
    return w32, x_bf16_as_f32.reshape(M, K)


def blas_info():
    """BLAS library, version and thread count numpy runs on, plus the host's CPU and thread variables."""
    info = {"cpu_count": os.cpu_count(), "machine": platform.machine()}
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    info["cpu_model"] = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        from threadpoolctl import threadpool_info
        b = [i for i in threadpool_info() if i.get("user_api") == "blas"]
        if b:
            info["blas"] = {"library": b[0].get("internal_api"), "version": b[0].get("version"),
                            "threads": b[0].get("num_threads"), "architecture": b[0].get("architecture")}
    except Exception:  # noqa: BLE001
        pass
    info["thread_env"] = {v: os.environ[v] for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
                          if v in os.environ}
    return info


def blas_threads():
    b = blas_info().get("blas") or {}
    return int(b.get("threads") or os.cpu_count())


def time_cpu_port(w32, x, budget_s=10.0, max_iters=5000, min_iters=20):
    from oracle.moe_oracle import linear
    linear(x, w32)  # warm
    t0 = time.perf_counter()
    it = 0
    while it < max_iters and (it < min_iters or time.perf_counter() - t0 < budget_s):
        linear(x, w32)
        it += 1
    dt = (time.perf_counter() - t0) / it
    return dt, it


def time_cpu_dequant(raw, rows=1024):
    """The reference's load-time step, gguf_dequant.dequantize (single-threaded
    numpy, restated in oracle/), timed on the first `rows` rows of the weight
    and scaled per byte to the whole weight: returns seconds for all N rows."""
    from oracle import gguf_dequant_oracle as O
    rb = (K // 256) * 144
    rows = min(rows, N)
    part = bytes(raw[: rows * rb])
    t0 = time.perf_counter()
    O.dequantize(part, QTYPE, (rows, K))
    return (time.perf_counter() - t0) * (N / rows)


def cpu_dequant_fields(raw, dt_matmul):
    """The three CPU figures: dequantize alone, the fp32 matmul alone (the
    `value`), and the two back to back (a path that dequantizes per call)."""
    t_deq = time_cpu_dequant(raw)
    return {"dequant": {"GBps": round(W_BYTES / t_deq / 1e9, 5), "s_per_weight": round(t_deq, 3), "threads": 1,
                        "sample": f"1024 of {N} rows, scaled per byte"},
            "dequant_plus_matmul": {"GBps": round(W_BYTES / (t_deq + dt_matmul) / 1e9, 5),
                                    "note": "per call if the weight were dequantized every step; the reference "
                                            "dequantizes once at load, so its per-step cost is the matmul"}}


def bf16_row(seed=1):
    """The activation row: N(0,1) rounded to bf16 (as fp32 values)."""
    x = np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)
    return (x.view(np.uint32) >> 16 << 16).view(np.float32)


# ---------------------------------------------------------------------------
def dist_setup(backend):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def run_reference(args):
    """The reference's CPU path of the same workload (fp32 x @ W.T on the weight it dequantized at
    load, ops.py:62-67 after gguf_dequant.py:309-341, restated in oracle/), all BLAS threads; one
    step = the row through the 16 weights of a step (one dequantized weight multiplied 16 times: at
    180 MB it is far out of every CPU cache either way).  Exactly K steps are timed for `value`;
    `sustained` repeats steps for at least ~2 s."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.moe_oracle import linear
    from xanosmerks_b200.synth import make_weight
    raw = make_weight(QTYPE, N, K, seed=0)
    w32, x = cpu_port_setup(raw, bf16_row())

    def step():
        for _ in range(COPIES):
            linear(x, w32)
    for _ in range(max(args.warmup, 3)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    v = COPIES * W_BYTES / dt / 1e9
    # and a run of at least ~2 s, so that a short K does not leave the figure to timer noise
    t0 = time.perf_counter()
    done = 0
    while done < 1 or time.perf_counter() - t0 < 2.0:
        step()
        done += 1
    t_sus = time.perf_counter() - t0
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config(),
           "reference_path": "numpy port of LinearOp.forward (ops.py:62-67) on the weight dequantized at load "
                             "(gguf_dequant.py:309-341), host CPU, all BLAS threads",
           "sustained": {"steps": done, "s": round(t_sus, 3),
                         "GBps": round(done * COPIES * W_BYTES / t_sus / 1e9, 3)},
           "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": blas_threads(), "kind": "port",
                            "sample": f"{args.steps} steps ({args.steps * COPIES} fp32 (1x{K}) @ ({K}x{N}) products) "
                                      f"after {max(args.warmup, 3)} warm-up steps",
                            "host": blas_info(), **cpu_dequant_fields(raw, dt / COPIES)},
           "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def graph_of(fn, count):
    """A CUDA graph of fn(0) .. fn(count - 1) (launches go to torch's current stream, the capture
    stream inside torch.cuda.graph)."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(count):
            fn(i)
    return g


def event_ms(run, stream=None):
    """Device time of run() with CUDA events on the current stream, synchronised on both sides."""
    import torch
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def time_rotating(fn, launches, warm=3):
    """Average device time (us) of fn(i) over `launches` graph-captured launches (fn rotates its own
    inputs over enough copies to keep them out of L2)."""
    for i in range(warm):
        fn(i)
    g = graph_of(fn, launches)
    g.replay()
    ms = event_ms(g.replay)
    del g
    return ms * 1e3 / launches


def copies_for(nbytes, floor=4):
    """Copies of an input so that one rotation is at least 4x the 126 MB L2."""
    return max(floor, math.ceil(4 * 126e6 / nbytes))


def gemv_configs(dev, peaks):
    """Config 1 (Q8_0 4096^2: dequant, and GEMV on fp32 x) and config 3 (Q6_K and Q5_K GEMV on
    4096^2, 4096x14336, 14336x4096 at batch 1 and 4, fp32 x), plus the standalone dequant kernel on
    the headline weight: weight GB/s and fraction of the measured HBM copy bandwidth."""
    import torch
    from xanosmerks_b200 import _lib
    from xanosmerks_b200.qtypes import normalize, row_bytes
    from xanosmerks_b200.synth import make_weight
    lib = _lib.lib
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    res = {"hbm_peak_GBps": hbm, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
           "l2_policy": "each input rotates over copies totalling >= 4x L2"}

    def weights(name, n, k, seed):
        wb = row_bytes(normalize(name), k) * n
        w0 = torch.from_numpy(make_weight(name, n, k, seed=seed)).to(dev)
        return [w0] + [w0.clone() for _ in range(copies_for(wb) - 1)], wb

    def gemv_point(name, n, k, m, ws_list, wb):
        qid = normalize(name).type_id
        x = torch.from_numpy(np.random.default_rng(3).standard_normal((m, k)).astype(np.float32)).to(dev)
        y = torch.empty((m, n), dtype=torch.float32, device=dev)
        wsz = lib.xm_qgemv_workspace_size(k, m)
        work = torch.empty(max(wsz, 16), dtype=torch.uint8, device=dev)

        def f(i):
            w = ws_list[i % len(ws_list)]
            _lib.check(lib.xm_qgemv(qid, w.data_ptr(), wb, n, k, x.data_ptr(), _lib.DT_F32, m, None, y.data_ptr(),
                                    work.data_ptr(), work.numel(), st()), "qgemv")
        us = time_rotating(f, max(64, 2 * len(ws_list)))
        gbps = wb / us / 1e3
        return {"us": round(us, 3), "weight_GBps": round(gbps, 1), "frac_of_hbm": round(gbps / hbm, 4)}

    # config 1: Q8_0 4096 x 4096
    ws_list, wb = weights("Q8_0", 4096, 4096, 31)
    c1 = {"weight_bytes": wb, "gemv_fp32_x_m1": gemv_point("Q8_0", 4096, 4096, 1, ws_list, wb)}
    out16 = torch.empty(4096 * 4096, dtype=torch.float16, device=dev)

    def deq(i):
        w = ws_list[i % len(ws_list)]
        _lib.check(lib.xm_dequantize(8, w.data_ptr(), wb, 4096 * 4096, out16.data_ptr(), _lib.DT_F16, st()),
                   "dequantize")
    us = time_rotating(deq, max(64, 2 * len(ws_list)))
    tot = wb + 4096 * 4096 * 2
    c1["dequant_f16"] = {"us": round(us, 3), "GBps_read_plus_write": round(tot / us / 1e3, 1),
                         "frac_of_hbm": round(tot / us / 1e3 / hbm, 4), "bytes": tot}
    res["q8_0_4096x4096"] = c1
    del ws_list, out16
    # standalone dequant of the headline Q4_K weight (fp16 out)
    ws_list, wb = weights("Q4_K", N, K, 33)
    o16 = torch.empty(N * K, dtype=torch.float16, device=dev)

    def deq4(i):
        w = ws_list[i % len(ws_list)]
        _lib.check(lib.xm_dequantize(12, w.data_ptr(), wb, N * K, o16.data_ptr(), _lib.DT_F16, st()), "dequantize")
    us = time_rotating(deq4, max(48, 2 * len(ws_list)))
    tot = wb + N * K * 2
    res["q4_k_dequant_11008x4096_f16"] = {"us": round(us, 3), "GBps_read_plus_write": round(tot / us / 1e3, 1),
                                          "frac_of_hbm": round(tot / us / 1e3 / hbm, 4), "bytes": tot}
    del ws_list, o16
    # config 3: Q6_K and Q5_K decode shapes
    for name in ("Q6_K", "Q5_K"):
        for n, k in ((4096, 4096), (4096, 14336), (14336, 4096)):
            ws_list, wb = weights(name, n, k, 35)
            pts = {f"m{m}": gemv_point(name, n, k, m, ws_list, wb) for m in (1, 4)}
            res[f"{name.lower()}_{n}x{k}"] = {"weight_bytes": wb, **pts}
            del ws_list
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist
    rank, world, local = dist_setup("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from xanosmerks_b200 import _lib
    from xanosmerks_b200.ops import GGUFTensor, LinearOp
    from xanosmerks_b200.synth import make_weight
    lib = _lib.lib
    qid = 12
    peaks = load_peaks()

    raw = make_weight(QTYPE, N, K, seed=rank)
    w0 = torch.from_numpy(raw).to(dev)
    ws = [w0] + [w0.clone() for _ in range(COPIES - 1)]
    xb = bf16_row()
    x_dev = torch.from_numpy(xb).to(dev).to(torch.bfloat16)
    wsz = lib.xm_qgemv_workspace_size(K, M)
    work = torch.empty(wsz, dtype=torch.uint8, device=dev)
    y = torch.empty((COPIES, M, N), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def launch(c):
        _lib.check(lib.xm_qgemv(qid, ws[c].data_ptr(), W_BYTES, N, K, x_dev.data_ptr(), _lib.DT_BF16, M, None,
                                y[c].data_ptr(), work.data_ptr(), wsz, torch.cuda.current_stream().cuda_stream),
                   "qgemv")

    def step(i):                       # the row through the 16 weights
        for c in range(COPIES):
            launch(c)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    g_steps = graph_of(step, args.steps)
    g_steps.replay()
    torch.cuda.synchronize()

    def timed(graph, reps=1):
        if world > 1:
            dist.barrier()
        ms = event_ms(lambda: [graph.replay() for _ in range(reps)], stream)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    with Clocks(local) as clk:
        ms_steps = timed(g_steps)
        # sustained: the same graph replayed for at least ~20 ms
        reps = max(1, math.ceil(20.0 / max(ms_steps, 1e-3)))
        ms_sus = timed(g_steps, reps)
    clocks = clk.summary()
    launches = args.steps * COPIES
    sustained = {"replays": reps, "steps": reps * args.steps, "launches": reps * launches, "ms": round(ms_sus, 3),
                 "GBps": round(world * reps * launches * W_BYTES / (ms_sus / 1e3) / 1e9, 1)}

    # correctness of the timed kernels: every weight's output of the last replay against the oracle
    from oracle import gguf_dequant_oracle as O
    wref = O.dequantize(raw, QTYPE, (N, K)).astype(np.float32)
    yref = (xb @ wref.T).astype(np.float64)
    yg = y.cpu().numpy().astype(np.float64)
    den = np.abs(yref).max()
    norm_err = float(np.abs(yg - yref).max() / den)
    elem_err = float((np.abs(yg - yref) / (np.abs(yref) + 1e-3 * den)).max())
    check = {"against": "oracle fp32 x @ W.T on the reference's fp16 weights (gguf_dequant.py:309-341)",
             "max_abs_err_over_max_ref": norm_err, "tolerance": 1e-3,
             "max_elementwise_rel_err": elem_err,
             "elementwise_definition": "|y - ref| / (|ref| + 1e-3 max|ref|), all 16 outputs of the last step",
             "pass": norm_err < 1e-3}

    # prefill sweep of the same weight (tensor-core dequant-GEMM) plus the M = 8 decode point: TFLOPS per M
    sweep = {}
    if not args.no_sweep:
        for mm in (8, 64, 512, 2048):
            xs = torch.from_numpy(np.random.default_rng(5).standard_normal((mm, K)).astype(np.float32)).to(dev).to(
                torch.bfloat16)
            ys = torch.empty((mm, N), dtype=torch.float32, device=dev)
            if mm > 8:
                gsz = lib.xm_qgemm_workspace_size_n(mm, N, K)
            else:
                gsz = lib.xm_qgemv_workspace_size(K, mm)
            gws = torch.empty(gsz, dtype=torch.uint8, device=dev)

            def gstep(i, xs=xs, ys=ys, gws=gws, gsz=gsz, mm=mm):
                w = ws[i % COPIES]
                fn = lib.xm_qgemm if mm > 8 else lib.xm_qgemv
                _lib.check(fn(qid, w.data_ptr(), W_BYTES, N, K, xs.data_ptr(), _lib.DT_BF16, mm, None, ys.data_ptr(),
                              gws.data_ptr(), gsz, torch.cuda.current_stream().cuda_stream), "qgemm")
            reps_g = 64 if mm <= 64 else (32 if mm <= 512 else 16)
            for i in range(3):
                gstep(i)
            g = graph_of(gstep, reps_g)
            g.replay()
            torch.cuda.synchronize()
            ms = timed(g)
            del g
            flops = 2.0 * mm * N * K
            tf = flops * reps_g / (ms / 1e3) / 1e12
            us = ms * 1e3 / reps_g
            sweep[f"M={mm}"] = {"TFLOPS": round(tf, 1), "us": round(us, 2),
                                "kernel": "tcgen05 GEMM (CTA pairs, decoded weights in tensor memory)" if mm > 8 else "integer mma.sync GEMV",
                                "frac_of_measured_bf16_peak": round(tf / float(peaks.get("bf16_tflops", 1590.0)), 4),
                                "weight_GBps": round(W_BYTES / us / 1e3, 1)}

    # end to end through the public API: pinned host activation in, fp32 result back to host, every call
    ops = [LinearOp(GGUFTensor(w, QTYPE, (N, K))) for w in ws]
    x_pin = torch.from_numpy(xb).to(torch.bfloat16).pin_memory()
    e2e_steps = max(2, min(args.steps, 20))
    for c in range(COPIES):
        ops[c].forward(x_pin)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for c in range(COPIES):
            out = ops[c].forward(x_pin)
    t_e2e = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([t_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_e2e = float(t.item())
    assert tuple(out.shape) == (M, N)
    e2e = {"value": round(world * e2e_steps * COPIES * W_BYTES / t_e2e / 1e9, 3), "unit": UNIT,
           "h2d_bytes_per_step": COPIES * M * K * 2, "d2h_bytes_per_step": COPIES * M * N * 4,
           "api": "xanosmerks_b200.ops.LinearOp(GGUFTensor).forward(pinned bf16 host tensor), one call per weight",
           "ms_per_step": round(t_e2e / e2e_steps * 1e3, 4), "us_per_call": round(t_e2e / e2e_steps / COPIES * 1e6, 2)}

    value = world * launches * W_BYTES / (ms_steps / 1e3) / 1e9
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    alg_bytes = W_BYTES + M * K * 2 + M * N * 4          # blocks + bf16 x + fp32 y
    avg_gemv_s = ms_steps / 1e3 / launches
    achieved = alg_bytes / avg_gemv_s / 1e9
    roofline = {"bound": "hbm", "kernel": KERNEL, "achieved": round(achieved, 1),
                "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": NCU_TRAFFIC_PER_LAUNCH, "algorithmic_bytes_per_launch": alg_bytes,
                "avg_launch_us": round(avg_gemv_s * 1e6, 3)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        w32, xc = cpu_port_setup(raw, xb)
        dt, it = time_cpu_port(w32, xc)
        cpu = {"value": round(W_BYTES / dt / 1e9, 3), "unit": UNIT, "cores": blas_threads(), "kind": "port",
               "sample": f"{it} fp32 (1x{K}) @ ({K}x{N}) products on the dequantized weight (~10 s)",
               "host": blas_info(), **cpu_dequant_fields(raw, dt)}

    configs = None if (args.no_configs or world > 1) else gemv_configs(dev, peaks)
    decode = None if args.no_decode else decode_section(args, rank, world, dev, peaks)
    moe = None if args.no_moe else (moe_section(dev, peaks) if world == 1 else moe_ep_section(dev, rank, world))

    if rank == 0:
        out = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms_steps / args.steps, 6), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "i32 dp4a + f32", "data": "synthetic",
               "config": config(), "check": check, "e2e": e2e, "roofline": roofline, "sustained": sustained,
               "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": launches,
               "prefill_sweep": {"metric": f"{QTYPE} {N}x{K} dequant-GEMM TFLOPS (bf16 x, fp16-exact weights)",
                                 "points": sweep},
               "configs": configs, "decode": decode, "moe": moe}
        print(json.dumps(out), flush=True)
    del g_steps
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def decode_section(args, rank, world, dev, peaks):
    """Llama decode tok/s (32 layers, d 4096, GQA 32/8, FFN 14336, vocab 32000;
    Q4_K attention and gate/up, Q6_K down and output): prompt of 512 random ids,
    then greedy decode steps replayed from a CUDA graph.  With N ranks the model
    is tensor-parallel over all of them (the row-parallel partial sums are
    all-reduced over NVLink peer memory), so per-step work is fixed as N grows
    (strong scaling)."""
    import torch
    import torch.distributed as dist
    from xanosmerks_b200.llama import LlamaConfig, LlamaDecoder, LlamaWeights, synth_llama_weights
    cfg = LlamaConfig()
    full = synth_llama_weights(cfg, seed=11, device=dev)
    weights = LlamaWeights.from_full(cfg, full, rank, world)
    del full
    torch.cuda.empty_cache()
    bpt = cfg.weight_bytes_per_token()
    res = {"model": "Llama 32L d4096 GQA32/8 FFN14336 V32000 (Q4_K attn+gate/up, Q6_K down+output; random-init)",
           "prompt": 512, "tensor_parallel": world, "weight_bytes_per_token": bpt, "points": {},
           "note": "prefill_512 = the 512-token prompt of every sequence through all layers into the KV cache "
                   "plus the first token; projection_TFLOPS counts the layer projections only"}
    steps = max(16, min(args.decode_steps, 120))
    st = torch.cuda.current_stream(dev)
    D, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    qkv_n = (cfg.num_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
    proj_flops_per_token = 2 * cfg.num_layers * D * (qkv_n + cfg.num_heads * cfg.head_dim + 2 * F) + \
        2 * cfg.num_layers * F * D
    for B in (1, 8):
        dec = LlamaDecoder(weights, batch=B, max_ctx=640)
        ids = torch.from_numpy(np.random.default_rng(12).integers(0, cfg.vocab_size, size=(B, 512)))
        dec.prefill(ids)                      # warm-up (allocations, tensor maps)
        dec.reset()
        if world > 1:
            dist.barrier()
        ms_pf = event_ms(lambda: dec.prefill(ids), st)
        if world > 1:
            t = torch.tensor([ms_pf], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_pf = float(t.item())
        pf_tf = proj_flops_per_token * B * 512 / (ms_pf / 1e3) / 1e12
        prefill = {"ms": round(ms_pf, 3), "tok_s": round(B * 512 / (ms_pf / 1e3), 1),
                   "projection_TFLOPS": round(pf_tf, 1),
                   "frac_of_measured_bf16_peak": round(pf_tf / float(peaks.get("bf16_tflops", 1590.0)), 4),
                   "path": "every projection over all B*512 rows on the tcgen05 GEMM (fused RMSNorm / SwiGLU / "
                           "residual), causal GQA attention of the whole prompt on tensor cores (one call per layer), split-K where the output tiles are few, output head on the last token"}
        dec.decode_step()
        dec.length += 1
        dec.capture()
        dec.replay(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        dec.replay(steps)
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        ms_tok = ms / steps
        # end to end: each step's token ids come from pinned host memory and the next ids go back to it
        pin_in = torch.zeros(B, dtype=torch.int32).pin_memory()
        pin_out = torch.zeros(B, dtype=torch.int32).pin_memory()
        pin_in.copy_(dec.next_ids.cpu())
        e2e_steps = min(steps, 640 - dec.length - 1)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            dec.next_ids.copy_(pin_in, non_blocking=True)
            dec.replay(1)
            pin_out.copy_(dec.next_ids, non_blocking=True)
            st.synchronize()
            pin_in.copy_(pin_out)
        t_e2e = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([t_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        gbps = bpt / world / (ms_tok / 1e3) / 1e9
        res["points"][f"batch{B}"] = {
            "tok_s": round(B * 1000.0 / ms_tok, 1), "ms_per_step": round(ms_tok, 4),
            "weight_GBps_per_gpu": round(gbps, 1),
            "hbm_frac_of_measured": round(gbps / float(peaks.get("hbm_gbs", 6650.0)), 4),
            "e2e_tok_s": round(B * e2e_steps / t_e2e, 1), "e2e_h2d_bytes_per_step": 4 * B,
            "e2e_d2h_bytes_per_step": 4 * B, "prefill_512": prefill}
        dec.close()
        del dec
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    del weights
    torch.cuda.empty_cache()
    return res


def moe_ep_section(dev, rank, world, T=1024, E=8, k=2, H=4096, F=14336, seed=0):
    """Mixtral-shape block with experts sharded over the ranks (E / N each) and
    T tokens per rank exchanged with all-to-all (weak scaling: tokens per rank
    fixed); the same seeded weights as the single-GPU section."""
    import torch
    import torch.distributed as dist
    from xanosmerks_b200.moe import MoELayerEP
    from xanosmerks_b200.ops import GGUFTensor
    from xanosmerks_b200.synth import make_weight
    rng = np.random.default_rng(seed)
    gate = rng.standard_normal((E, H)).astype(np.float32) * 0.02
    weights = {"gate": {"weight": gate}, "experts": {}}
    el = E // world
    for e in range(rank * el, (rank + 1) * el):
        weights["experts"][str(e)] = {
            wn: {"weight": GGUFTensor(make_weight("Q4_K", *shape, seed=seed * 1000 + 3 * e + i), "Q4_K", shape,
                                      device=dev)}
            for i, (wn, shape) in enumerate((("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))))}
    layer = MoELayerEP({"num_experts": E, "num_experts_per_tok": k, "hidden_act": "silu"}, weights, rank, world)
    x = torch.from_numpy(np.random.default_rng(100 + rank).standard_normal((T, H)).astype(np.float32)).to(dev).to(
        torch.bfloat16)
    for _ in range(2):
        layer.forward_device(x)
    torch.cuda.synchronize()
    dist.barrier()
    reps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        layer.forward_device(x)
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / reps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    del layer
    torch.cuda.empty_cache()
    flops = 2.0 * T * world * k * 3 * F * H
    return {"block": f"Mixtral-shape MoE, expert-parallel over {world} GPUs ({E // world} experts each), "
                     f"{T} bf16 tokens per GPU, NCCL all-to-all exchange, Q4_K experts",
            "us": round(us, 1), "TFLOPS_total": round(flops / us / 1e6, 1),
            "tokens_per_s": round(T * world / us * 1e6, 1), "scaling": "weak"}


def moe_section(dev, peaks):
    import torch
    layer, x, flops = moe_case(dev)
    for _ in range(2):
        layer.forward_device(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        layer.forward_device(x)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    del layer
    torch.cuda.empty_cache()
    tf = flops / us / 1e6
    return {"block": "Mixtral-shape MoE, 8 experts top-2, 1024 bf16 tokens, 4096->14336 SwiGLU, Q4_K experts",
            "us": round(us, 1), "TFLOPS": round(tf, 1), "tokens_per_s": round(1024 / us * 1e6, 1),
            "frac_of_measured_bf16_peak": round(tf / float(peaks.get("bf16_tflops", 1590.0)), 4)}


def _profile_weight(args, dev):
    from xanosmerks_b200.qtypes import normalize, row_bytes
    from xanosmerks_b200.synth import make_weight
    import torch
    qt = normalize(args.gemm_type)
    n, k = args.gemm_n, args.gemm_k
    wb = row_bytes(qt, k) * n
    w0 = torch.from_numpy(make_weight(qt.name, n, k, seed=0)).to(dev)
    copies = min(copies_for(wb, 2), 16)
    return qt, n, k, wb, [w0] + [w0.clone() for _ in range(copies - 1)]


def run_gemm_only(args):
    """One prefill GEMM shape (--gemm-type, --gemm-n x --gemm-k, --gemm-m rows of bf16 x), timed
    alone; the mode ncu captures use."""
    import torch
    from xanosmerks_b200 import _lib
    lib = _lib.lib
    dev = torch.device("cuda", 0)
    qt, n, k, wb, ws = _profile_weight(args, dev)
    mm = args.gemm_m
    xs = torch.from_numpy(np.random.default_rng(5).standard_normal((mm, k)).astype(np.float32)).to(dev).to(torch.bfloat16)
    ys = torch.empty((mm, n), dtype=torch.float32, device=dev)
    gsz = lib.xm_qgemm_workspace_size_n(mm, n, k)
    gws = torch.empty(gsz, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def call(i):
        _lib.check(lib.xm_qgemm(qt.type_id, ws[i % len(ws)].data_ptr(), wb, n, k, xs.data_ptr(), _lib.DT_BF16, mm,
                                None, ys.data_ptr(), gws.data_ptr(), gsz, st), "qgemm")
    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        e0.record()
        for i in range(args.steps):
            call(i)
        e1.record()
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"gemm": qt.name, "m": mm, "n": n, "k": k, "us": round(us, 2),
                      "TFLOPS": round(2.0 * mm * n * k / us / 1e6, 1), "clocks": clk.summary()}), flush=True)


def run_gemv_only(args):
    """--gemv-only launches of the decode GEMV (--gemm-type, --gemm-n x --gemm-k, --gemv-m fp32 rows)."""
    import torch
    from xanosmerks_b200 import _lib
    lib = _lib.lib
    dev = torch.device("cuda", 0)
    qt, n, k, wb, ws = _profile_weight(args, dev)
    m = args.gemv_m
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((m, k)).astype(np.float32)).to(dev)
    y = torch.empty((m, n), dtype=torch.float32, device=dev)
    wsz = max(16, lib.xm_qgemv_workspace_size(k, m))
    work = torch.empty(wsz, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def call(i):
        _lib.check(lib.xm_qgemv(qt.type_id, ws[i % len(ws)].data_ptr(), wb, n, k, x.data_ptr(), _lib.DT_F32, m, None,
                                y.data_ptr(), work.data_ptr(), wsz, st), "qgemv")
    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    ms = event_ms(lambda: [call(i) for i in range(args.gemv_only)])
    us = ms * 1e3 / args.gemv_only
    print(json.dumps({"gemv": qt.name, "m": m, "n": n, "k": k, "us": round(us, 3),
                      "weight_GBps": round(wb / us / 1e3, 1)}), flush=True)


def run_dequant_only(args):
    """--dequant-only launches of the standalone dequant kernel (--gemm-type, --gemm-n x --gemm-k, fp16 out)."""
    import torch
    from xanosmerks_b200 import _lib
    lib = _lib.lib
    dev = torch.device("cuda", 0)
    qt, n, k, wb, ws = _profile_weight(args, dev)
    out = torch.empty(n * k, dtype=torch.float16, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def call(i):
        _lib.check(lib.xm_dequantize(qt.type_id, ws[i % len(ws)].data_ptr(), wb, n * k, out.data_ptr(), _lib.DT_F16,
                                     st), "dequantize")
    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    ms = event_ms(lambda: [call(i) for i in range(args.dequant_only)])
    us = ms * 1e3 / args.dequant_only
    print(json.dumps({"dequant": qt.name, "n": n, "k": k, "us": round(us, 3),
                      "GBps_read_plus_write": round((wb + 2 * n * k) / us / 1e3, 1)}), flush=True)


def run_decode_profile(args):
    """Profiling mode: the bench's Llama shapes with --decode-layers layers, an
    8-token prompt, one eager decode step, then two replays of the captured
    step between cudaProfilerStart and cudaProfilerStop."""
    import torch
    from xanosmerks_b200.llama import LlamaConfig, LlamaDecoder, LlamaWeights, synth_llama_weights
    B = args.decode_profile
    cfg = LlamaConfig(num_layers=args.decode_layers)
    w = LlamaWeights.from_full(cfg, synth_llama_weights(cfg, seed=0, device="cuda"))
    dec = LlamaDecoder(w, batch=B, max_ctx=640)
    ids = np.random.default_rng(0).integers(0, cfg.vocab_size, size=(B, 8))
    dec.prefill(torch.from_numpy(ids))
    dec.decode_step()
    dec.length += 1
    dec.capture()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    dec.replay(2)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"decode_profile": B, "layers": args.decode_layers, "ok": True}), flush=True)


def run_prefill_profile(args):
    """Profiling mode: the bench's Llama shapes with --decode-layers layers; one warm-up prefill of a
    --prefill-profile-token prompt (batch 1), then a second one between cudaProfilerStart/Stop."""
    import torch
    from xanosmerks_b200.llama import LlamaConfig, LlamaDecoder, LlamaWeights, synth_llama_weights
    cfg = LlamaConfig(num_layers=args.decode_layers)
    w = LlamaWeights.from_full(cfg, synth_llama_weights(cfg, seed=0, device="cuda"))
    dec = LlamaDecoder(w, batch=1, max_ctx=640)
    ids = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab_size, size=(1, args.prefill_profile)))
    dec.prefill(ids)
    dec.reset()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    ms = event_ms(lambda: dec.prefill(ids))
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"prefill_profile": args.prefill_profile, "layers": args.decode_layers, "ms": round(ms, 3)}),
          flush=True)


def moe_case(dev, T=1024, E=8, k=2, H=4096, F=14336, seed=0):
    """Mixtral-shape MoE block with random-init Q4_K experts (seeded)."""
    import torch
    from xanosmerks_b200.moe import MoELayer
    from xanosmerks_b200.ops import GGUFTensor
    from xanosmerks_b200.synth import make_weight
    rng = np.random.default_rng(seed)
    gate = rng.standard_normal((E, H)).astype(np.float32) * 0.02
    weights = {"gate": {"weight": gate}, "experts": {}}
    for e in range(E):
        weights["experts"][str(e)] = {
            wn: {"weight": GGUFTensor(make_weight("Q4_K", *shape, seed=seed * 1000 + 3 * e + i), "Q4_K", shape,
                                      device=dev)}
            for i, (wn, shape) in enumerate((("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))))}
    layer = MoELayer({"num_experts": E, "num_experts_per_tok": k, "hidden_act": "silu"}, weights)
    x = torch.from_numpy(rng.standard_normal((1, T, H)).astype(np.float32)).to(dev).to(torch.bfloat16)
    flops = 2.0 * T * k * 3 * F * H
    return layer, x, flops


def run_moe_only(args):
    import torch
    dev = torch.device("cuda", 0)
    layer, x, flops = moe_case(dev)
    for _ in range(args.warmup):
        layer.forward_device(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        e0.record()
        for _ in range(args.steps):
            layer.forward_device(x)
        e1.record()
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"moe": "Mixtral-shape block, 8 experts top-2, 1024 tokens, 4096->14336 Q4_K",
                      "us": round(us, 1), "TFLOPS": round(flops / us / 1e6, 1),
                      "tokens_per_s": round(1024 / us * 1e6, 1), "clocks": clk.summary()}), flush=True)


def main():
    args = parse()
    if args.moe:
        run_moe_only(args)
        return
    if args.decode_profile:
        run_decode_profile(args)
        return
    if args.prefill_profile:
        run_prefill_profile(args)
        return
    if args.gemm_m:
        run_gemm_only(args)
        return
    if args.gemv_only:
        run_gemv_only(args)
        return
    if args.dequant_only:
        run_dequant_only(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
