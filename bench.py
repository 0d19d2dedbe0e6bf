"""Benchmark of the EXL3 quantized-linear hot path on B200 (one JSON line on rank 0).

Metric: "EXL3 GEMV effective HBM GB/s; batch-1 decode tok/s at 27B-class on 1/2/4/8 GPU".

Workload of one step (the decode GEMV sweep): every combination of the 27B-class
projection shapes 5120->17408, 17408->5120, 5120->6144, 5120->5120, bitrates K in {2,3,4,5,6,8} and
rows in {1,2,4,8}: 96 GEMV launches, 3inst codebook, seeded uniform trellis, +-1 svh, fp16 N(0,1)
activations (synthetic stand-ins for checkpoint tensors). Rows are the outer loop, so between two uses
of one weight matrix the other 23 matrices (~0.8 GB, > L2) stream through: every launch reads its
trellis from HBM. value = algorithmic bytes of all launches / device time of the step, where a launch's
algorithmic bytes are k*n*K/8 + rows*k*2 + n*2 + rows*n*2 (trellis, xh, svh, y).

With --gpus N (torchrun) every rank runs the same sweep on its own GPU (independent weight matrices,
no collective): weak scaling, value = total bytes of all ranks / max over ranks of the step time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own CPU path for this workload (its trellis decode source
compiled for the CPU by oracle/build_ref.py, an fp32 GEMV and the 128-point output rotation) on the
host cores, on a bounded sample of the same sweep; the reference's Metal path cannot run here.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPES = [(5120, 17408), (17408, 5120), (5120, 6144), (5120, 5120)]
BITS = [2, 3, 4, 5, 6, 8]
ROWS = [1, 2, 4, 8]


def select_case(spec: str | None):
    """--case k,n,K,rows narrows the sweep to one GEMV configuration (used for small ncu captures)."""
    global SHAPES, BITS, ROWS
    if spec:
        k, n, K, rows = (int(v) for v in spec.split(","))
        SHAPES, BITS, ROWS = [(k, n)], [K], [rows]
METRIC = "EXL3 GEMV effective HBM GB/s; batch-1 decode tok/s at 27B-class on 1/2/4/8 GPU"


def alg_bytes(k, n, K, rows):
    return k * n * K // 8 + rows * k * 2 + n * 2 + rows * n * 2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops_sustained", 1376.1)), "measured"
    return 6650.0, 1400.0, "fallback"


# ------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------ ours

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from omlx_exl3_b200 import EXL3Linear
    from omlx_exl3_b200.kernels import TrellisGemvPlan

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    # resident synthetic weights: one trellis / svh per (shape, K)
    mats = {}
    for (k, n) in SHAPES:
        for K in BITS:
            nwords = k * n * K // 32
            tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (nwords,), dtype=torch.int32, device=dev, generator=gen)
            svh = (torch.randint(0, 2, (n,), device=dev, generator=gen).to(torch.float16) * 2 - 1)
            mats[(k, n, K)] = (tr, svh)
    plans, xs = [], []
    for rows in ROWS:
        for (k, n) in SHAPES:
            for K in BITS:
                tr, svh = mats[(k, n, K)]
                plan = TrellisGemvPlan(k, [n], K, 0, svh, rows, torch.float16)
                xh = torch.randn((1, rows, k), device=dev, generator=gen).to(torch.float16)
                y = torch.empty((rows, n), dtype=torch.float16, device=dev)
                plans.append((plan, xh, tr, y, alg_bytes(k, n, K, rows), (k, n, K, rows)))
    step_bytes = sum(p[4] for p in plans)
    stream = torch.cuda.current_stream(dev)

    def step():
        for plan, xh, tr, y, _, _ in plans:
            plan(xh, [tr], out=y)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # The step's 96 launches are captured once in a CUDA graph, so the device runs them back to back
    # (host launch cost is not part of a kernel's time).
    step()
    torch.cuda.synchronize(dev)
    cap_stream = torch.cuda.Stream(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap_stream):
        with torch.cuda.graph(graph, stream=cap_stream):
            step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)

    # device time of a subset of the step's launches (one graph per bitrate / row count), for the
    # breakdown keys; a bitrate group re-reads each matrix 4 times (once per row count), so for
    # K <= 3 (< 126 MB of weights per group) part of those reads can come from L2
    def group_ms(idx):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap_stream):
            with torch.cuda.graph(g, stream=cap_stream):
                for i in idx:
                    plan, xh, tr, y, _, _ = plans[i]
                    plan(xh, [tr], out=y)
        g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(3):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / 3

    # timed region: K graph replays, CUDA events on the launching stream
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    t0.record(stream)
    for s in range(args.steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop()
    ms_total = t0.elapsed_time(t1)

    # ---- end to end through the public module API: host x -> EXL3Linear -> host y
    e2e = None
    if rank == 0 or world > 1:
        lins = []
        for (k, n) in SHAPES:
            for K in BITS:
                tr, svh = mats[(k, n, K)]
                lin = EXL3Linear(k, n, {"trellis": ((k // 16, n // 16, 16 * K), torch.int16),
                                         "suh": ((k,), torch.float16), "svh": ((n,), torch.float16)}, device=dev)
                lin.trellis.view(torch.int32).reshape(-1).copy_(tr)
                lin.suh.copy_(torch.ones(k, device=dev, dtype=torch.float16))
                lin.svh.copy_(svh)
                lins.append((lin, k, n, K))
        host_x = {(rows, k): torch.randn((rows, k), generator=None).to(torch.float16).pin_memory()
                  for rows in ROWS for k in {s[0] for s in SHAPES}}
        host_y = {(rows, n): torch.empty((rows, n), dtype=torch.float16).pin_memory()
                  for rows in ROWS for n in {s[1] for s in SHAPES}}
        h2d = d2h = 0

        def e2e_step():
            nonlocal h2d, d2h
            h2d = d2h = 0
            for rows in ROWS:
                for lin, k, n, K in lins:
                    xd = host_x[(rows, k)].to(dev, non_blocking=True)
                    yd = lin(xd)
                    host_y[(rows, n)].copy_(yd, non_blocking=True)
                    h2d += rows * k * 2
                    d2h += rows * n * 2
        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        e2e = (e2e_ms, h2d, d2h)

    # ---- max over ranks
    ms_step = ms_total / args.steps
    vals = torch.tensor([ms_step, e2e[0] if e2e else 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_step, e2e_ms = float(vals[0]), float(vals[1])
    if rank != 0:
        return None

    hbm_peak, _, peak_kind = load_peaks()
    launch_bytes = np.array([p[4] for p in plans], dtype=np.float64)
    # every launch of the step is the GEMV kernel: the average launch moves step_bytes / n bytes in
    # ms_step / n, so the step's rate is the kernel's achieved rate
    achieved = float(launch_bytes.sum() / (ms_step * 1e-3) / 1e9)
    per_k, per_rows = {}, {}
    if len(BITS) > 1:
        for K in BITS:
            idx = [i for i, p in enumerate(plans) if p[5][2] == K]
            per_k[str(K)] = round(float(launch_bytes[idx].sum() / (group_ms(idx) * 1e-3) / 1e9), 1)
    if len(ROWS) > 1:
        for r in ROWS:
            idx = [i for i, p in enumerate(plans) if p[5][3] == r]
            per_rows[str(r)] = round(float(launch_bytes[idx].sum() / (group_ms(idx) * 1e-3) / 1e9), 1)
    value = step_bytes * world / (ms_step * 1e-3) / 1e9
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded uniform trellis, +-1 svh, fp16 N(0,1) activations)",
        "config": {"workload": "BASELINE config 2: decode GEMV sweep, 4 shapes x K{2,3,4,5,6,8} x rows{1,2,4,8}, "
                               "3inst codebook (96 launches per step per GPU)",
                   "shapes": [f"{k}->{n}" for k, n in SHAPES], "bits": BITS, "rows": ROWS,
                   "l2": "inputs larger than L2: 24 matrices (~0.83 GB) cycle between two uses of one matrix",
                   "parallelism": f"replicas x{world} (independent matrices per GPU, no collective)"},
        "gemv_GBps_by_bits": per_k,
        "gemv_GBps_by_rows": per_rows,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4),
                     # per average launch: algorithmic bytes x the DRAM (read + write) / algorithmic
                     # ratio 1.0057 of the ncu capture in profiles/gemv_kernel_sweep.md
                     # (5120->17408, K=6, rows=1)
                     "traffic": round(float(launch_bytes.mean()) * 1.0057),
                     "traffic_unit": "bytes per launch",
                     "kernel": "exl3::gemv_kernel", "peak_kind": peak_kind,
                     "frac_of_8TBps_nominal": round(achieved / 8000.0, 4)},
        "clocks": clk,
        "gpu_launches": len(plans) * args.steps,
    }
    if e2e:
        out["e2e"] = {"value": round(step_bytes * world / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                      "h2d_bytes_per_step": e2e[1], "d2h_bytes_per_step": e2e[2],
                      "path": "EXL3Linear.forward (rot + GEMV) with pinned host x in and host y out"}
    return out


# ------------------------------------------------------------------------------------------ prefill

def run_prefill(args, local_rank):
    """prefill GEMM at 6 bpw, M in {512, 4096} x (5120->17408, 17408->5120), bf16
    output. The fused kernel (trellis decoded in shared memory, tcgen05 into tensor memory) and the
    decode-once path (exl3_decode_wt to fp16, a library fp16 GEMM, exl3_had_svh) are both timed with
    CUDA events; TFLOP/s counts 2*M*k*n."""
    import torch

    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.prefill import use_fused

    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    _, tf_peak, kind = load_peaks()
    rows = []
    for (k, n) in ((5120, 17408), (17408, 5120)):
        K = 6
        tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (k * n * K // 32,), dtype=torch.int32, device=dev, generator=gen)
        svh = (torch.randint(0, 2, (n,), device=dev, generator=gen).to(torch.float16) * 2 - 1)
        for M in (512, 4096):
            xh = torch.randn((M, k), device=dev, generator=gen).to(torch.float16)
            y = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
            wt = torch.empty((n, k), dtype=torch.float16, device=dev)
            yh = torch.empty((M, n), dtype=torch.float16, device=dev)

            def fused():
                kernels.gemm(xh, tr, k, n, K, 0, svh, torch.bfloat16, out=y)

            def decode_once():
                kernels.decode_wt(tr, k, n, K, 0, out=wt)
                torch.matmul(xh, wt.t(), out=yh)
                kernels.had_svh(yh, svh, torch.bfloat16)

            res = {"M": M, "k": k, "n": n, "bits": K,
                   "default": "fused_tcgen05" if use_fused(M, n) else "decode_once_gemm"}
            for name, fn in (("fused_tcgen05", fused), ("decode_once_gemm", decode_once)):
                for _ in range(3):
                    fn()
                torch.cuda.synchronize(dev)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                it = 10
                a.record()
                for _ in range(it):
                    fn()
                b.record()
                torch.cuda.synchronize(dev)
                ms = a.elapsed_time(b) / it
                tf = 2.0 * M * k * n / (ms * 1e-3) / 1e12
                res[name] = {"us": round(ms * 1000, 1), "TFLOPs": round(tf, 1), "frac": round(tf / tf_peak, 4)}
            rows.append(res)
            del xh, y, wt, yh
        del tr
    torch.cuda.empty_cache()
    return {"peak_TFLOPs": tf_peak, "peak_kind": f"{kind} bf16 sustained (fp16 has the same rate)",
            "status": kernels.gemm_status(dev), "cases": rows}


# ------------------------------------------------------------------------------------------ decode

def run_decode(args, rank, world, local_rank):
    """batch-1 decode of the random-init 64-layer 27B-class model (hidden 5120,
    40 q / 8 kv heads x 128, SwiGLU 17408, vocab 151936 with an 8-bpw EXL3 head, per-tensor bitrates
    5..8 averaging 6.0) over a 4096-token random fp16 KV cache, tensor-parallel over the `world` GPUs
    (NCCL all-reduce after o_proj and down_proj, logit arg-max gathered). One step = one token through
    the captured decode graph; tok/s = steps / max over ranks of the device time."""
    import torch
    import torch.distributed as dist

    from omlx_exl3_b200.decode import DecodeRunner
    from omlx_exl3_b200.loader import draw_bits, synthetic_model
    from omlx_exl3_b200.model import ModelConfig

    dev = torch.device("cuda", local_rank)
    cfg = ModelConfig(num_hidden_layers=args.decode_layers, max_position_embeddings=4200)
    bits = draw_bits(cfg.num_hidden_layers, seed=0, cfg=cfg)
    t_build = time.time()
    model = synthetic_model(cfg, bits, 8, tp_rank=rank, tp_size=world, device=dev, seed=0)
    cache = model.make_cache(4097)
    cache.fill_random(4096, seed=1 + rank)
    torch.cuda.synchronize(dev)
    t_build = time.time() - t_build
    runner = DecodeRunner(model, cache, rows=1, use_graph=True)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(3, args.warmup)):
        runner.step()
    torch.cuda.synchronize(dev)
    n = max(20, args.steps)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        runner.step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = e0.elapsed_time(e1) / n

    # end to end: the token goes in from (pinned) host memory and the next token comes back every step
    tok_host = torch.tensor([17], dtype=torch.long).pin_memory()
    out_host = torch.zeros(1, dtype=torch.long).pin_memory()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(n):
        nxt = runner.step(tok_host.to(dev, non_blocking=True))
        out_host.copy_(nxt, non_blocking=True)
    e3.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms_e2e = e2.elapsed_time(e3) / n

    vals = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    runner.release()
    peer_ar = model.tp.peers is not None
    if world > 1:
        barrier()
    model.close_peers()
    weights = sum(b.numel() * b.element_size() for m in model.modules() for nm, b in m.named_buffers(recurse=False)
                  if nm == "trellis")
    del runner, model, cache
    torch.cuda.empty_cache()
    ms, ms_e2e = float(vals[0]), float(vals[1])
    return {"tok_s": round(1000.0 / ms, 2), "ms_per_token": round(ms, 4), "tp": world, "steps": n,
            "allreduce": "fused NVLink peer kernel (exl3_ar_add_norm_rot)" if peer_ar else
                         ("NCCL" if world > 1 else "none"),
            "e2e_tok_s": round(1000.0 / ms_e2e, 2),
            "trellis_bytes_per_gpu": int(weights),
            "weight_stream_GBps_per_gpu": round(weights / (ms * 1e-3) / 1e9, 1),
            "build_s": round(t_build, 1),
            "model": f"random-init Qwen3-style, {cfg.num_hidden_layers} layers, hidden 5120, 40q/8kv x 128, "
                     "SwiGLU 17408, vocab 151936 (8-bpw EXL3 head), per-group bpw 5..8 averaging 6.0, "
                     "4096-token random fp16 KV cache, CUDA-graph decode step"}


# ------------------------------------------------------------------------------------------ CPU

def cpu_reference_sample(budget_s: float = 12.0):
    """The reference's CPU path (oracle/_ref: its decode source + fp32 GEMV + rotation) on a bounded
    sample of the sweep: one 5120->5120 GEMV per K at rows 1, repeated until ~budget_s seconds."""
    from oracle import oracle as O
    L = O.ref_lib()
    kind = "reference"
    if L is None:
        kind = "port"
    threads = os.cpu_count() or 1
    if L is not None:
        L.exl3_ref_set_threads(threads)
    else:
        O.lib().exl3o_set_threads(threads)
    rng = np.random.default_rng(0)
    k = n = 5120
    cases = []
    for K in BITS:
        t = O.random_trellis(k, n, K, 77 + K)
        xh = rng.standard_normal((1, k)).astype(np.float16)
        svh = np.where(rng.random(n) < 0.5, -1, 1).astype(np.float16)
        cases.append((K, t, xh, svh))
    done_bytes, t_start, calls = 0, time.perf_counter(), 0
    while True:
        for K, t, xh, svh in cases:
            if L is not None:
                y = np.empty((1, n), np.float32)
                L.exl3_ref_gemv(K, 0, O._ptr(O.trellis_u32(t)), k, n, O._ptr(xh.view(np.uint16)), 1,
                                O._ptr(svh.view(np.uint16)), O._ptr(y))
            else:
                O.gemv_c(t, k, n, K, 0, xh, svh)
            done_bytes += alg_bytes(k, n, K, 1)
            calls += 1
        if time.perf_counter() - t_start > budget_s:
            break
    dt = time.perf_counter() - t_start
    return {"value": round(done_bytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{calls} GEMVs 5120->5120 rows 1, K in {BITS} (3inst), decode+fp32 GEMV+rotation, "
                      f"{dt:.1f} s on {threads} host threads"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    budget = max(3.0, min(20.0, 60.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_reference_sample(budget_s=0.5)
    samples = [cpu_reference_sample(budget_s=budget) for _ in range(args.steps)]
    v = float(np.median([s["value"] for s in samples]))
    cpu = dict(samples[-1])
    cpu["value"] = v
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": v,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": None,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded uniform trellis, +-1 svh, fp16 N(0,1) activations)",
        "config": {"workload": "BASELINE config 2 decode GEMV sweep, bounded CPU sample (5120->5120, rows 1, "
                               "K in {2,3,4,5,6,8})",
                   "note": "reference Metal path unavailable on this box; CPU = reference decode source "
                           "compiled by oracle/build_ref.py + fp32 GEMV + FWHT"},
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", default=None, help="k,n,K,rows: one GEMV configuration instead of the sweep")
    ap.add_argument("--no-decode", action="store_true", help="skip the 27B-class TP decode measurement")
    ap.add_argument("--decode-layers", type=int, default=64)
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill GEMM measurement")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the TP decode measurement (prints its own JSON line; for profiling the step)")
    args = ap.parse_args()
    select_case(args.case)
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        if args.decode_only:
            dec = run_decode(args, rank, world, local_rank)
            if rank == 0:
                print(json.dumps({"metric": "decode_tok_s", "value": dec["tok_s"], "unit": "tok/s", "n_gpus": world,
                                  "decode": dec}), flush=True)
            return
        out = run_ours(args, rank, world, local_rank)
        dec = None if (args.no_decode or args.case) else run_decode(args, rank, world, local_rank)
        pre = run_prefill(args, local_rank) if (world == 1 and not args.case and not args.no_prefill) else None
        if out is not None:
            if dec is not None:
                out["decode"] = dec
            if pre is not None:
                out["prefill_gemm"] = pre
            if world == 1 and not args.no_cpu_baseline:
                out["cpu_baseline"] = cpu_reference_sample(budget_s=12.0)
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
