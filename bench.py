#!/usr/bin/env python
"""Benchmark of the quantized-weight decode path: Q4_K GEMV weight GB/s.

Workload: W = 11008 x 4096 in GGUF Q4_K (25,362,432 bytes of blocks), one bf16
activation row (M = 1), fp32 output -- the decode point of the Q4_K
dequant-GEMM sweep.  One step = one call of the fused dequant-GEMV on one
weight matrix (a single kernel: the activation split happens in its prologue).  Steps rotate over 16
distinct weight copies (406 MB, more than 3x the 126 MB L2), so every step
streams its weight from HBM.  Weights and activations are seeded synthetic
data (random-init blocks with the documented value distributions).

Printed line (rank 0): ``value`` = quantized weight bytes of all steps of all
ranks / max-over-ranks device time of the timed graph replay; ``e2e`` = the
same metric through the public ``LinearOp.forward`` with the activation coming
from pinned host memory and the result read back every step; ``roofline`` =
the GEMV kernel alone against the measured HBM copy bandwidth;
``cpu_baseline`` = the numpy restatement of the reference's path (fp32 x @ W.T
on the dequantized weight) on this host's cores.

``--impl reference`` times the reference's CPU path (the numpy port in
``oracle/``) on the same workload instead.  Multi-GPU (torchrun): every rank
runs the same per-GPU workload on its own weights (weak scaling; the row
blocks are independent, so there is no collective in the data path).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

QTYPE, N, K, M = "Q4_K", 11008, 4096, 1
W_BYTES = N * (K // 256) * 144          # 25,362,432
COPIES = 16
METRIC = "Q4_K GEMV weight GB/s"
UNIT = "GB/s"
# DRAM bytes read+written per launch of the GEMV kernel on this shape, from the
# ncu capture summarised in profiles/q4k_gemv_k4096_m1_11008x4096.md.
NCU_TRAFFIC_PER_LAUNCH = 25_409_536
KERNEL = "k_qgemv_q4k_k4096_m1<bf16> (fused activation split)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the prefill (tensor-core GEMM) sweep")
    ap.add_argument("--moe", action="store_true",
                    help="only time the Mixtral-shape MoE block (8 experts, top-2, 1024 tokens, 4096 -> 14336)")
    ap.add_argument("--no-decode", action="store_true", help="skip the Llama decode tok/s section")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE block section")
    ap.add_argument("--decode-steps", type=int, default=64)
    ap.add_argument("--decode-profile", type=int, default=0,
                    help="profiling mode: two graph-replayed decode steps of this batch size between "
                         "cudaProfilerStart/Stop (with --decode-layers layers)")
    ap.add_argument("--decode-layers", type=int, default=2)
    ap.add_argument("--gemm-m", type=int, default=0,
                    help="only time the prefill GEMM with this many activation rows (profiling mode)")
    return ap.parse_args()


def config(extra=None):
    c = {"workload": f"{QTYPE} GEMV {N}x{K}, M={M}, bf16 activations, fp32 out",
         "weight_bytes": W_BYTES, "weight_copies": COPIES,
         "l2_policy": f"inputs larger than L2: {COPIES} rotating weight copies = {COPIES * W_BYTES / 1e6:.0f} MB",
         "parallelism": "independent replicas per GPU (row blocks), no collective"}
    if extra:
        c.update(extra)
    return c


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


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(n[0]) if n else os.cpu_count()
    except Exception:  # noqa: BLE001
        return os.cpu_count()


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
    rank, world, local = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0
    if rank != 0:
        return
    from xanosmerks_b200.synth import make_weight
    raw = make_weight(QTYPE, N, K, seed=0)
    xb = (np.random.default_rng(1).standard_normal((M, K)).astype(np.float32).view(np.uint32) >> 16 << 16).view(np.float32)
    w32, x = cpu_port_setup(raw, xb)
    from oracle.moe_oracle import linear
    for _ in range(args.warmup):
        linear(x, w32)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        linear(x, w32)
        ts.append(time.perf_counter() - t0)
    dt = sum(ts) / len(ts)
    v = W_BYTES / dt / 1e9
    cores = blas_threads()
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": config({"reference_path": "numpy port of LinearOp.forward (ops.py:62-67) on the weight "
                                               "dequantized at load (gguf_dequant.py:309-341), host CPU"}),
           "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": cores, "kind": "port",
                            "sample": f"{args.steps} steps of fp32 (1x{K}) @ ({K}x{N}) numpy/BLAS",
                            **cpu_dequant_fields(raw, dt)},
           "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


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

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    raw = make_weight(QTYPE, N, K, seed=rank)
    w0 = torch.from_numpy(raw).to(dev)
    ws = [w0] + [w0.clone() for _ in range(COPIES - 1)]
    xb = (np.random.default_rng(1).standard_normal((M, K)).astype(np.float32).view(np.uint32) >> 16 << 16).view(np.float32)
    x_dev = torch.from_numpy(xb).to(dev).to(torch.bfloat16)
    wsz = lib.xm_qgemv_workspace_size(K, M)
    work = torch.empty(wsz, dtype=torch.uint8, device=dev)
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    # launches go to torch's current stream, which is the capture stream inside torch.cuda.graph
    def step(i):
        w = ws[i % COPIES]
        _lib.check(lib.xm_qgemv(qid, w.data_ptr(), W_BYTES, N, K, x_dev.data_ptr(), _lib.DT_BF16, M, None,
                                y.data_ptr(), work.data_ptr(), wsz, torch.cuda.current_stream().cuda_stream), "qgemv")

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()

    def capture(fn, count):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(count):
                fn(i)
        return g

    g_steps = capture(step, args.steps)
    for _ in range(2):
        g_steps.replay()
    torch.cuda.synchronize()

    def timed(graph):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    with Clocks(local) as clk:
        ms_steps = timed(g_steps)
    clocks = clk.summary()
    ms_gemv = ms_steps          # one kernel per step

    # correctness guard on the last result (rank-local, cheap): exact path on the same weight
    y_exact = torch.empty_like(y)
    w_last = ws[(args.steps - 1) % COPIES]
    _lib.check(lib.xm_qgemv_exact(qid, w_last.data_ptr(), W_BYTES, N, K, x_dev.data_ptr(), _lib.DT_BF16, M, None,
                                  y_exact.data_ptr(), stream.cuda_stream), "qgemv_exact")
    g_steps.replay()
    torch.cuda.synchronize()
    err = float((y - y_exact).abs().max() / y_exact.abs().max())

    # prefill sweep of the same weight (tensor-core dequant-GEMM): TFLOPS per M
    sweep = {}
    if not args.no_sweep:
        for mm in (64, 512, 2048):
            xs = torch.from_numpy(np.random.default_rng(5).standard_normal((mm, K)).astype(np.float32)).to(dev).to(
                torch.bfloat16)
            ys = torch.empty((mm, N), dtype=torch.float32, device=dev)
            gsz = lib.xm_qgemm_workspace_size(mm, K)
            gws = torch.empty(gsz, dtype=torch.uint8, device=dev)

            def gstep(i, xs=xs, ys=ys, gws=gws, gsz=gsz, mm=mm):
                w = ws[i % COPIES]
                _lib.check(lib.xm_qgemm(qid, w.data_ptr(), W_BYTES, N, K, xs.data_ptr(), _lib.DT_BF16, mm, None,
                                        ys.data_ptr(), gws.data_ptr(), gsz,
                                        torch.cuda.current_stream().cuda_stream), "qgemm")
            reps = 50 if mm <= 512 else 20
            for i in range(3):
                gstep(i)
            g = capture(gstep, reps)
            g.replay()
            torch.cuda.synchronize()
            ms = timed(g)
            del g
            flops = 2.0 * mm * N * K
            tf = flops * reps / (ms / 1e3) / 1e12
            sweep[f"M={mm}"] = {"TFLOPS": round(tf, 1), "us": round(ms * 1e3 / reps, 2),
                                "frac_of_measured_bf16_peak": round(tf / float(peaks.get("bf16_tflops", 1590.0)), 4)}

    # end to end through the public API: pinned host activation in, fp32 result back to host, every step
    ops = [LinearOp(GGUFTensor(w, QTYPE, (N, K))) for w in ws]
    x_pin = torch.from_numpy(xb).to(torch.bfloat16).pin_memory()
    e2e_steps = min(args.steps, 200)
    for i in range(5):
        ops[i % COPIES].forward(x_pin)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        out = ops[i % COPIES].forward(x_pin)
    t_e2e = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([t_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_e2e = float(t.item())
    assert out.shape == (M, N)
    e2e = {"value": round(world * e2e_steps * W_BYTES / t_e2e / 1e9, 3), "unit": UNIT,
           "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 4,
           "api": "xanosmerks_b200.ops.LinearOp(GGUFTensor).forward(pinned bf16 host tensor)",
           "ms_per_step": round(t_e2e / e2e_steps * 1e3, 4)}

    value = world * args.steps * W_BYTES / (ms_steps / 1e3) / 1e9
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    alg_bytes = W_BYTES + M * K * 2 + M * N * 4          # blocks + bf16 x + fp32 y
    avg_gemv_s = ms_gemv / 1e3 / args.steps
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
               "sample": f"{it} steps of fp32 (1x{K}) @ ({K}x{N}) numpy/BLAS on the dequantized weight (~10 s)",
               **cpu_dequant_fields(raw, dt)}

    decode = None if args.no_decode else decode_section(args, rank, world, dev, peaks)
    moe = None if args.no_moe else (moe_section(dev) if world == 1 else moe_ep_section(dev, rank, world))

    if rank == 0:
        out = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms_steps / args.steps, 6), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "i32 dp4a + f32", "data": "synthetic",
               "config": config({"max_rel_err_vs_exact_path": err}), "e2e": e2e, "roofline": roofline,
               "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": args.steps,
               "prefill_sweep": {"metric": f"{QTYPE} {N}x{K} dequant-GEMM TFLOPS (bf16 x, fp16-exact weights)",
                                 "points": sweep},
               "decode": decode, "moe": moe}
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
           "prompt": 512, "tensor_parallel": world, "weight_bytes_per_token": bpt, "points": {}}
    steps = max(16, min(args.decode_steps, 120))
    st = torch.cuda.current_stream(dev)
    for B in (1, 8):
        dec = LlamaDecoder(weights, batch=B, max_ctx=640)
        ids = torch.from_numpy(np.random.default_rng(12).integers(0, cfg.vocab_size, size=(B, 512)))
        dec.prefill(ids)
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
            "e2e_d2h_bytes_per_step": 4 * B}
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


def moe_section(dev):
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
    return {"block": "Mixtral-shape MoE, 8 experts top-2, 1024 bf16 tokens, 4096->14336 SwiGLU, Q4_K experts",
            "us": round(us, 1), "TFLOPS": round(flops / us / 1e6, 1), "tokens_per_s": round(1024 / us * 1e6, 1)}


def run_gemm_only(args):
    """One prefill GEMM shape, timed alone (the mode ncu captures use)."""
    import torch
    from xanosmerks_b200 import _lib
    from xanosmerks_b200.synth import make_weight
    lib = _lib.lib
    dev = torch.device("cuda", 0)
    w = torch.from_numpy(make_weight(QTYPE, N, K, seed=0)).to(dev)
    mm = args.gemm_m
    xs = torch.from_numpy(np.random.default_rng(5).standard_normal((mm, K)).astype(np.float32)).to(dev).to(torch.bfloat16)
    ys = torch.empty((mm, N), dtype=torch.float32, device=dev)
    gsz = lib.xm_qgemm_workspace_size(mm, K)
    gws = torch.empty(gsz, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        _lib.check(lib.xm_qgemm(12, w.data_ptr(), W_BYTES, N, K, xs.data_ptr(), _lib.DT_BF16, mm, None,
                                ys.data_ptr(), gws.data_ptr(), gsz, st), "qgemm")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        e0.record()
        for _ in range(args.steps):
            _lib.check(lib.xm_qgemm(12, w.data_ptr(), W_BYTES, N, K, xs.data_ptr(), _lib.DT_BF16, mm, None,
                                    ys.data_ptr(), gws.data_ptr(), gsz, st), "qgemm")
        e1.record()
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"gemm_m": mm, "n": N, "k": K, "us": round(us, 2),
                      "TFLOPS": round(2.0 * mm * N * K / us / 1e6, 1), "clocks": clk.summary()}), flush=True)


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
    if args.gemm_m:
        run_gemm_only(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
