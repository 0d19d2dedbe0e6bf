"""Benchmark of the EXL3 quantized-linear hot path on B200 (one JSON line on rank 0).

Metric: "EXL3 GEMV effective HBM GB/s; batch-1 decode tok/s at 27B-class on 1/2/4/8 GPU".

value: batch-1 decode tok/s of the 27B-class model of BASELINE config 5 (64 layers, hidden 5120, 40 q /
8 kv heads x 128, SwiGLU 17408, vocab 151936 with an 8-bpw EXL3 head, per-tensor bitrates 5..8 bpw
averaging 6.0, a 4096-token random fp16 KV cache; seeded random-init weights generated on the device),
tensor-parallel over the N GPUs of the run: strong scaling, the same model at every N, so the driver's
efficiency over N is the tensor-parallel decode's. One step is one token through the CUDA-graph-captured
decode step; the step streams all ~17 GB of weights, far more than L2, so no step reads another's
weights from cache. Time = CUDA events on the launching stream, max over ranks.

Beside it in the same line:
  e2e            the same tok/s through decode.DecodeRunner.step with the token copied in from pinned
                 host memory and the greedy next token copied back every step
  roofline       the dominant kernel of the step, the EXL3 GEMV: the step's GEMV launches replayed on
                 their own (same plans and buffers), algorithmic bytes per launch / mean launch time
                 (N = 1); plus the whole step's bytes per token / time per token
  gemv_sweep     BASELINE config 2 (the GEMV GB/s half of the metric): 4 shapes x K{2,3,4,5,6,8} x
                 rows{1,2,4,8}, 96 launches in one graph; GB/s per bitrate with the HBM and the
                 instruction-issue (ALU) fractions, and the same sweep end to end through EXL3Linear
  config1        BASELINE config 1 (4096->4096, 4 bpw, batch 1) on the GPU and, same config, on the CPU
  layer          BASELINE config 4: one decoder layer (no head) at this N
  verify         the 4-token MTP-verify step (rows = 4) of the config-5 model at this N
  tp_parity      N > 1: logits of a 2-layer model of the same shapes, tensor-parallel vs unsharded
  prefill_gemm   BASELINE config 3 (N = 1)
  cpu_baseline   the reference's CPU path (its own decode source compiled for the host by
                 oracle/build_ref.py, fp32 GEMV, output rotation) timed on the host cores on a bounded
                 sample of the decode workload, extrapolated to tok/s (N = 1, rank 0)

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own CPU implementation of the path (the Metal path cannot run
here) on the same decode workload and config 1, rank 0 only.
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

METRIC = "EXL3 GEMV effective HBM GB/s; batch-1 decode tok/s at 27B-class on 1/2/4/8 GPU"
SWEEP_SHAPES = [(5120, 17408), (17408, 5120), (5120, 6144), (5120, 5120)]
SWEEP_BITS = [2, 3, 4, 5, 6, 8]
SWEEP_ROWS = [1, 2, 4, 8]
KV_LEN = 4096

# Warp instructions per 16x16 trellis tile of the GEMV kernel, per bitrate (rows = 1, 5120 -> 17408,
# one launch each): smsp__inst_executed.sum / (k * n / 256) from an ncu capture of the current kernel.
# Used for the instruction-issue (ALU) roofline of the sweep; a bitrate without a capture gets none.
INST_PER_TILE: dict[int, float] = {2: 43.6, 3: 48.9, 4: 41.5, 5: 48.8, 6: 46.8, 8: 39.7}
ISSUE_PER_SM_CYCLE = 4                 # warp instructions issued per SM per cycle (4 schedulers)


def gemv_bytes(k, ns, Ks, rows, out_bytes=2):
    """Algorithmic bytes of one GEMV launch: trellis + rotated inputs + svh + outputs."""
    nm, n = len(ns), sum(ns)
    return sum(k * nn * K // 8 for nn, K in zip(ns, Ks)) + nm * rows * k * 2 + n * 2 + rows * n * out_bytes


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "tf_burst": float(d.get("bf16_tflops", 1590.0)),
                "tf_sustained": float(d.get("bf16_tflops_sustained", 1400.0)),
                "sm_mhz": float(d.get("sm_max_mhz", 1965.0)), "kind": "measured"}
    return {"hbm": 6650.0, "tf_burst": 1590.0, "tf_sustained": 1400.0, "sm_mhz": 1965.0, "kind": "fallback"}


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


# ------------------------------------------------------------------------------------------ helpers

class LaunchCounter:
    """Counts the package's kernel launches (calls of the C ABI's launching entry points) while active."""

    LAUNCHING = ("exl3_gemv", "exl3_gemv_qkv_post", "exl3_gemv_peer", "exl3_rot", "exl3_norm_rot",
                 "exl3_swiglu_rot", "exl3_add_norm_rot", "exl3_ar_add_norm_rot", "exl3_attn_decode_rot",
                 "exl3_argmax", "exl3_qkv_post", "exl3_peer_put", "exl3_gemm", "exl3_decode_wt", "exl3_had_svh")
    # entry points that launch two kernels
    DOUBLE = ("exl3_attn_decode_rot",)

    def __init__(self):
        from omlx_exl3_b200 import _lib
        self.L = _lib.lib()
        self.count = 0
        self.orig = {}

    def __enter__(self):
        for name in self.LAUNCHING:
            fn = getattr(self.L, name)
            self.orig[name] = fn
            n = 2 if name in self.DOUBLE else 1

            def wrap(*a, _fn=fn, _n=n):
                self.count += _n
                return _fn(*a)
            setattr(self.L, name, wrap)
        return self

    def __exit__(self, *exc):
        for name, fn in self.orig.items():
            setattr(self.L, name, fn)


class GemvRecorder:
    """Records the GEMV launches (TrellisGemvPlan calls) of one eager pass, to replay them alone."""

    def __init__(self):
        from omlx_exl3_b200.kernels import TrellisGemvPlan
        self.cls = TrellisGemvPlan
        self.calls = []
        self.orig = {}

    def __enter__(self):
        for meth in ("__call__", "qkv_post", "peer"):
            fn = getattr(self.cls, meth)
            self.orig[meth] = fn

            def wrap(plan, *a, _fn=fn, **kw):
                self.calls.append((plan, _fn, a, kw))
                return _fn(plan, *a, **kw)
            setattr(self.cls, meth, wrap)
        return self

    def __exit__(self, *exc):
        for meth, fn in self.orig.items():
            setattr(self.cls, meth, fn)

    def bytes_of(self, plan) -> int:
        return gemv_bytes(plan.k, plan.member_ns, plan.Ks, plan.rows)

    def replay(self):
        for plan, fn, a, kw in self.calls:
            fn(plan, *a, **kw)


def time_graph(torch, dev, fn, reps: int, stream=None) -> float:
    """ms per replay of fn captured in a CUDA graph (CUDA events on the replay stream)."""
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        fn()
        with torch.cuda.graph(g, stream=cap):
            fn()
    torch.cuda.current_stream(dev).wait_stream(cap)
    s = torch.cuda.current_stream(dev)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(reps):
        g.replay()
    b.record(s)
    torch.cuda.synchronize(dev)
    del g
    return a.elapsed_time(b) / reps


# ------------------------------------------------------------------------------------------ decode

def model_cfg(layers: int):
    from omlx_exl3_b200.model import ModelConfig
    return ModelConfig(num_hidden_layers=layers, max_position_embeddings=KV_LEN + 104)


def build_model(torch, layers, rank, world, dev, head_bits=8, seed=0):
    from omlx_exl3_b200.loader import draw_bits, synthetic_model
    cfg = model_cfg(layers)
    bits = draw_bits(64, seed=0, cfg=cfg)[:layers]
    return synthetic_model(cfg, bits, head_bits, tp_rank=rank, tp_size=world, device=dev, seed=seed)


def kv_cache_for(model, full_seed: int, dev, length=KV_LEN, extra=16):
    """The model's KV cache holding this rank's kv heads of one seeded full-width random cache, so every
    tensor-parallel size sees the same cache contents."""
    import torch
    cfg, tp = model.cfg, model.tp
    cache = model.make_cache(length + extra)
    hkv_local = cfg.num_key_value_heads // tp.size
    h0 = tp.rank * hkv_local
    g = torch.Generator(device=dev)
    for i in range(cfg.num_hidden_layers):
        for dst in (cache.k[i], cache.v[i]):
            g.manual_seed(full_seed * 1000 + i * 2 + (dst is cache.v[i]))
            full = torch.randn((cfg.num_key_value_heads, length, cfg.head_dim), device=dev, generator=g)
            dst[:, :length].copy_(full[h0:h0 + hkv_local])
    cache.length = length
    return cache


def run_decode(args, torch, dist, rank, world, dev, layers=64, rows=1, head=True, gemv_roofline=False,
               timed_steps=None):
    """Decode steps of the config-5 model (or `layers` layers) at this tensor-parallel size: device tok/s
    (max over ranks), the e2e rate through DecodeRunner.step with host token in/out, launches per step
    and (gemv_roofline) the step's GEMV launches replayed alone."""
    from omlx_exl3_b200.decode import DecodeRunner

    t0 = time.time()
    model = build_model(torch, layers, rank, world, dev, head_bits=8 if head else None)
    cache = kv_cache_for(model, 1, dev)
    torch.cuda.synchronize(dev)
    build_s = time.time() - t0
    runner = DecodeRunner(model, cache, rows=rows, use_graph=True, check_every=0)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])

    steps = timed_steps or args.steps
    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev.index)
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        runner.step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop() if rank == 0 else None
    ms = e0.elapsed_time(e1) / steps

    # end to end: the token(s) come from pinned host memory, the greedy next token(s) go back each step
    tok_host = torch.full((rows,), 17, dtype=torch.long).pin_memory()
    out_host = torch.zeros(rows, dtype=torch.long).pin_memory()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(steps):
        nxt = runner.step(tok_host.to(dev, non_blocking=True))
        out_host.copy_(nxt, non_blocking=True)
    e3.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms_e2e = e2.elapsed_time(e3) / steps
    runner.check()                  # bounded waits of the peer all-reduce: raise if one ever gave up

    # launches per step: one eager pass of the step counted at the C ABI
    with LaunchCounter() as lc:
        runner._run()
    launches_per_step = lc.count
    torch.cuda.synchronize(dev)

    gemv = None
    if gemv_roofline and world == 1:
        rec = GemvRecorder()
        with rec:
            runner._run()
        torch.cuda.synchronize(dev)
        n_calls = len(rec.calls)
        gbytes = sum(rec.bytes_of(c[0]) for c in rec.calls)
        ms_g = time_graph(torch, dev, rec.replay, reps=max(3, steps))
        gemv = {"launches": n_calls, "bytes_per_launch": int(gbytes / n_calls),
                "us_per_launch": round(ms_g * 1000 / n_calls, 2),
                "achieved_GBps": round(gbytes / (ms_g * 1e-3) / 1e9, 1),
                "share_of_step": round(ms_g / ms, 3)}

    vals = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(vals[0]), float(vals[1])
    runner.release()
    peer_ar = model.tp.peers is not None
    barrier()
    model.close_peers()
    trellis = sum(b.numel() * b.element_size() for m in model.modules() for nm, b in m.named_buffers(recurse=False)
                  if nm == "trellis")
    cfg = model.cfg
    kv_bytes = 2 * cfg.num_hidden_layers * (KV_LEN + rows) * (cfg.num_key_value_heads // world) * cfg.head_dim * 2
    del runner, model, cache
    torch.cuda.empty_cache()
    return {"tok_s": round(rows * 1000.0 / ms, 2), "ms_per_step": round(ms, 4), "rows": rows, "tp": world,
            "steps": steps, "e2e_tok_s": round(rows * 1000.0 / ms_e2e, 2), "ms_per_step_e2e": round(ms_e2e, 4),
            "allreduce": "fused NVLink peer kernel (exl3_gemv_peer + exl3_ar_add_norm_rot)" if peer_ar else
                         ("NCCL" if world > 1 else "none"),
            "launches_per_step": launches_per_step, "bytes_per_step_per_gpu": int(trellis + kv_bytes),
            "step_GBps_per_gpu": round((trellis + kv_bytes) / (ms * 1e-3) / 1e9, 1), "build_s": round(build_s, 1),
            "gemv": gemv, "clocks": clk}


def run_timeline(args, torch, dist, rank, world, dev, layers=8, rows=1):
    """Per-kernel critical-path breakdown of the graph-replayed decode step at this tensor-parallel size.

    CUPTI kernel records (torch.profiler) of the last of three replays are sorted by start; each kernel is
    charged the time by which it moves the step's end (its end minus the latest end before it), so the
    increments sum to the step's span and overlapped work (a dependent launch's prologue, the weight
    prefetch) costs nothing. Rank 0 prints one JSON line: per kernel kind launches per layer, increment
    per layer and mean duration."""
    import collections
    from torch.profiler import ProfilerActivity, profile
    from omlx_exl3_b200.decode import DecodeRunner

    model = build_model(torch, layers, rank, world, dev)
    cache = kv_cache_for(model, 1, dev)
    runner = DecodeRunner(model, cache, rows=rows, use_graph=True, check_every=0)
    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        runner.step()
    e1.record()
    torch.cuda.synchronize(dev)
    us_layer = e0.elapsed_time(e1) * 1000.0 / args.steps / layers
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(3):
            runner.step()
        torch.cuda.synchronize(dev)
    runner.check()
    ks = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                if e.device_type.name == "CUDA")
    ks = ks[-(len(ks) // 3):]
    inc, dur, cnt = collections.defaultdict(float), collections.defaultdict(float), collections.Counter()
    prev_end = ks[0][0]
    for st, en, name in ks:
        kind = name.split("(")[0].replace("void ", "")
        inc[kind] += max(0.0, en - prev_end)
        dur[kind] += en - st
        cnt[kind] += 1
        prev_end = max(prev_end, en)
    runner.release()
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    model.close_peers()
    if rank != 0:
        return None
    kinds = sorted(inc, key=lambda k: -inc[k])
    return {"timeline": {"tp": world, "layers": layers, "rows": rows, "us_per_layer_graph": round(us_layer, 2),
                         "profiled_step_us": round(ks[-1][1] - ks[0][0], 1),
                         "kernels": [{"kernel": k, "launches_per_layer": round(cnt[k] / layers, 3),
                                      "increment_us_per_layer": round(inc[k] / layers, 2),
                                      "us_per_launch": round(dur[k] / cnt[k], 2)} for k in kinds]}}


def run_tp_parity(torch, dist, rank, world, dev, layers=2):
    """Logits of one decode step of a `layers`-layer model of the config-5 shapes, tensor-parallel over
    the group (fused peer all-reduce, logits gathered) against the same model unsharded on this rank.
    Returns {kl, argmax_equal, max_abs_logit_diff} on rank 0 (KL of the unsharded softmax to the TP one)."""
    from omlx_exl3_b200.decode import DecodeRunner
    tok = torch.tensor([1234], dtype=torch.long, device=dev)

    def one_step(tp_rank, tp_size):
        model = build_model(torch, layers, tp_rank, tp_size, dev, head_bits=8, seed=5)
        cache = kv_cache_for(model, 3, dev)
        runner = DecodeRunner(model, cache, rows=1, use_graph=False, check_every=0)
        local = runner.model(tok, cache, runner.pos)
        logits = model.gather_logits(local).float() if tp_size > 1 else local[:, :model.cfg.vocab_size].float()
        runner.check()
        torch.cuda.synchronize(dev)
        if tp_size > 1:
            dist.barrier(device_ids=[dev.index])
        model.close_peers()
        del runner, model, cache
        return logits

    tp_logits = one_step(rank, world)
    ref_logits = one_step(0, 1)
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    lp_ref = torch.log_softmax(ref_logits.clamp_min(-200), -1)
    lp_tp = torch.log_softmax(tp_logits.clamp_min(-200), -1)
    kl = float((lp_ref.exp() * (lp_ref - lp_tp)).sum(-1).max())
    return {"kl": kl, "argmax_equal": bool(torch.equal(ref_logits.argmax(-1), tp_logits.argmax(-1))),
            "max_abs_logit_diff": round(float((ref_logits - tp_logits).abs().max()), 5),
            "layers": layers, "kl_tolerance": 1e-4, "ok": kl <= 1e-4}


# ------------------------------------------------------------------------------------------ GEMV

def run_sweep(args, torch, dev, peaks):
    """the decode GEMV sweep in one CUDA graph; GB/s by bitrate / rows; HBM and
    instruction-issue fractions; the same sweep end to end through EXL3Linear.forward."""
    from omlx_exl3_b200 import EXL3Linear
    from omlx_exl3_b200.kernels import TrellisGemvPlan

    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    mats = {}
    for (k, n) in SWEEP_SHAPES:
        for K in SWEEP_BITS:
            tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (k * n * K // 32,), dtype=torch.int32, device=dev, generator=gen)
            svh = (torch.randint(0, 2, (n,), device=dev, generator=gen).to(torch.float16) * 2 - 1)
            mats[(k, n, K)] = (tr, svh)
    plans = []
    for rows in SWEEP_ROWS:                        # rows outermost: ~0.8 GB of other matrices between reuses
        for (k, n) in SWEEP_SHAPES:
            for K in SWEEP_BITS:
                tr, svh = mats[(k, n, K)]
                plan = TrellisGemvPlan(k, [n], K, 0, svh, rows, torch.float16)
                xh = torch.randn((1, rows, k), device=dev, generator=gen).to(torch.float16)
                y = torch.empty((rows, n), dtype=torch.float16, device=dev)
                plans.append((plan, xh, tr, y, gemv_bytes(k, [n], [K], rows), (k, n, K, rows)))

    def run(idx):
        def f():
            for i in idx:
                plan, xh, tr, y, _, _ = plans[i]
                plan(xh, [tr], out=y)
        return f

    allidx = list(range(len(plans)))
    reps = max(3, args.steps)
    ms = time_graph(torch, dev, run(allidx), reps)
    total = sum(p[4] for p in plans)
    by_bits, by_rows = {}, {}
    clock = peaks["sm_mhz"]
    for K in SWEEP_BITS:
        idx = [i for i, p in enumerate(plans) if p[5][2] == K]
        b = sum(plans[i][4] for i in idx)
        t = time_graph(torch, dev, run(idx), reps)
        weights = sum(plans[i][5][0] * plans[i][5][1] for i in idx)
        ent = {"GBps": round(b / (t * 1e-3) / 1e9, 1), "hbm_frac": round(b / (t * 1e-3) / 1e9 / peaks["hbm"], 4),
               "weights_per_s": float(f"{weights / (t * 1e-3):.4g}")}
        if INST_PER_TILE.get(K):
            inst_rate = weights / 256 * INST_PER_TILE[K] / (t * 1e-3)          # warp instructions / s
            inst_peak = 148 * ISSUE_PER_SM_CYCLE * clock * 1e6
            ent.update(alu_frac=round(inst_rate / inst_peak, 4), inst_per_tile=INST_PER_TILE[K])
        by_bits[str(K)] = ent
    for r in SWEEP_ROWS:
        idx = [i for i, p in enumerate(plans) if p[5][3] == r]
        b = sum(plans[i][4] for i in idx)
        by_rows[str(r)] = round(b / (time_graph(torch, dev, run(idx), reps) * 1e-3) / 1e9, 1)

    # the same matrices read as the mcg and mul1 codebooks (same bytes, other hash constants; the
    # reference's kernel test runs all three), rows 1 and 4, GB/s per codebook
    by_codebook = {}
    for cb, name in ((0, "3inst"), (1, "mcg"), (2, "mul1")):
        cplans = []
        for rows in (1, 4):
            for (k, n) in SWEEP_SHAPES:
                for K in SWEEP_BITS:
                    tr, svh = mats[(k, n, K)]
                    plan = TrellisGemvPlan(k, [n], K, cb, svh, rows, torch.float16)
                    xh = torch.randn((1, rows, k), device=dev, generator=gen).to(torch.float16)
                    y = torch.empty((rows, n), dtype=torch.float16, device=dev)
                    cplans.append((plan, xh, tr, y, gemv_bytes(k, [n], [K], rows)))

        def crun():
            for plan, xh, tr, y, _ in cplans:
                plan(xh, [tr], out=y)
        t = time_graph(torch, dev, crun, reps)
        by_codebook[name] = round(sum(c[4] for c in cplans) / (t * 1e-3) / 1e9, 1)
        del cplans

    # end to end through the module: pinned host x in, host y out, EXL3Linear.forward (rotation + GEMV)
    lins = []
    for (k, n) in SWEEP_SHAPES:
        for K in SWEEP_BITS:
            tr, svh = mats[(k, n, K)]
            lin = EXL3Linear(k, n, {"trellis": ((k // 16, n // 16, 16 * K), torch.int16),
                                     "suh": ((k,), torch.float16), "svh": ((n,), torch.float16)}, device=dev)
            lin.trellis.view(torch.int32).reshape(-1).copy_(tr)
            lin.suh.fill_(1.0)
            lin.svh.copy_(svh)
            lins.append((lin, k, n))
    host_x = {(r, k): torch.randn((r, k)).to(torch.float16).pin_memory() for r in SWEEP_ROWS for k in {5120, 17408}}
    host_y = {(r, n): torch.empty((r, n), dtype=torch.float16).pin_memory() for r in SWEEP_ROWS
              for n in {s[1] for s in SWEEP_SHAPES}}
    moved = [0, 0]
    # The module calls run on the compute stream; each call's input copy runs on an upload stream and
    # its output copy on a download stream, ordered by events, so the transfers overlap the neighbouring
    # calls' GEMVs as in a pipelined caller instead of sitting between the kernels of one stream. Every
    # call has its own device input buffer, whose upload waits for the previous step's GEMV that read it.
    stream = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    calls = [(lin, k, n, r) for r in SWEEP_ROWS for lin, k, n in lins]
    dev_x = [torch.empty((r, k), dtype=torch.float16, device=dev) for (_, k, _, r) in calls]
    ev_in = [torch.cuda.Event() for _ in calls]
    ev_done = [torch.cuda.Event() for _ in calls]
    ev_done_used = [False] * len(calls)

    def e2e_step():
        moved[0] = moved[1] = 0
        up.wait_stream(stream)                                  # a step's transfers start inside its timing
        for i, (lin, k, n, r) in enumerate(calls):
            with torch.cuda.stream(up):
                if ev_done_used[i]:
                    up.wait_event(ev_done[i])
                dev_x[i].copy_(host_x[(r, k)], non_blocking=True)
                ev_in[i].record(up)
            stream.wait_event(ev_in[i])
            yd = lin(dev_x[i])
            ev_done[i].record(stream)
            ev_done_used[i] = True
            down.wait_event(ev_done[i])
            with torch.cuda.stream(down):
                host_y[(r, n)].copy_(yd, non_blocking=True)
            yd.record_stream(down)
            moved[0] += r * k * 2
            moved[1] += r * n * 2
        stream.wait_stream(down)                                # the step ends when its last output is home
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms_e2e = a.elapsed_time(b) / reps
    achieved = total / (ms * 1e-3) / 1e9
    out = {"workload": "BASELINE config 2: 4 shapes x K{2,3,4,5,6,8} x rows{1,2,4,8}, 3inst, 96 launches per step",
           "GBps": round(achieved, 1), "ms_per_step": round(ms, 4), "accumulate": "fp32",
           "hbm_frac": round(achieved / peaks["hbm"], 4), "by_bits": by_bits, "by_rows": by_rows,
           "by_codebook_rows_1_4": by_codebook,
           "e2e_GBps": round(total / (ms_e2e * 1e-3) / 1e9, 1),
           "e2e_path": "EXL3Linear.forward (rotation + GEMV) per call, pinned host x copied in on an upload "
                       "stream and y copied out to pinned host memory on a download stream, event-ordered",
           "e2e_h2d_bytes_per_step": moved[0], "e2e_d2h_bytes_per_step": moved[1]}
    del plans, mats, lins
    torch.cuda.empty_cache()
    return out


def run_config1(args, torch, dev, peaks):
    """4096 -> 4096 at 4 bpw, batch 1, 3inst: device GEMV GB/s over 64 copies of the
    weight (> L2) and the e2e rate through EXL3Linear.forward with host x / y."""
    from omlx_exl3_b200 import EXL3Linear
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    k = n = 4096
    K = 4
    copies = 64                                        # 64 x 8.4 MB = 537 MB of trellis: larger than L2
    gen = torch.Generator(device=dev)
    gen.manual_seed(4096)
    trs = [torch.randint(-2 ** 31, 2 ** 31 - 1, (k * n * K // 32,), dtype=torch.int32, device=dev, generator=gen)
           for _ in range(copies)]
    svh = (torch.randint(0, 2, (n,), device=dev, generator=gen).to(torch.float16) * 2 - 1)
    plan = TrellisGemvPlan(k, [n], K, 0, svh, 1, torch.float16)
    xh = torch.randn((1, 1, k), device=dev, generator=gen).to(torch.float16)
    y = torch.empty((1, n), dtype=torch.float16, device=dev)

    def f():
        for t in trs:
            plan(xh, [t], out=y)
    ms = time_graph(torch, dev, f, max(3, args.steps)) / copies
    b = gemv_bytes(k, [n], [K], 1)
    lin = EXL3Linear(k, n, {"trellis": ((k // 16, n // 16, 16 * K), torch.int16), "suh": ((k,), torch.float16),
                            "svh": ((n,), torch.float16)}, device=dev)
    lin.trellis.view(torch.int32).reshape(-1).copy_(trs[0])
    lin.suh.fill_(1.0)
    lin.svh.copy_(svh)
    hx = torch.randn((1, k)).to(torch.float16).pin_memory()
    hy = torch.empty((1, n), dtype=torch.float16).pin_memory()
    stream = torch.cuda.current_stream(dev)
    for _ in range(5):
        hy.copy_(lin(hx.to(dev, non_blocking=True)), non_blocking=True)
    torch.cuda.synchronize(dev)
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 200
    a.record(stream)
    for _ in range(reps):
        hy.copy_(lin(hx.to(dev, non_blocking=True)), non_blocking=True)
    e.record(stream)
    torch.cuda.synchronize(dev)
    ms_e2e = a.elapsed_time(e) / reps
    del trs
    torch.cuda.empty_cache()
    return {"workload": "BASELINE config 1: 4096->4096, 4 bpw, batch 1, 3inst, +-1 svh",
            "GBps": round(b / (ms * 1e-3) / 1e9, 1), "us": round(ms * 1000, 2),
            "hbm_frac": round(b / (ms * 1e-3) / 1e9 / peaks["hbm"], 4),
            "e2e_GBps": round(b / (ms_e2e * 1e-3) / 1e9, 1), "e2e_us": round(ms_e2e * 1000, 2),
            "e2e_path": "EXL3Linear.forward with pinned host x in and host y out, one call per step"}


# ------------------------------------------------------------------------------------------ prefill

def run_prefill(args, torch, dev, peaks):
    """prefill GEMM at 6 bpw, M in {512, 4096} x (5120->17408, 17408->5120), bf16 out.
    Side by side: the fused kernel (trellis decoded in shared memory), decode-once + this package's
    tcgen05 GEMM on the decoded weights, the same GEMM alone (its own tensor-core rate), and decode-once +
    the library GEMM + had_svh (cuBLAS, a comparison only: never shipped). `default` is what
    prefill.linear_prefill runs. TFLOP/s counts 2*M*k*n; each call is timed alone, so the fraction is of the
    burst bf16 peak."""
    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.prefill import use_fused

    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    tf_peak = peaks["tf_burst"]
    cases = []
    for (k, n) in ((5120, 17408), (17408, 5120)):
        K = 6
        tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (k * n * K // 32,), dtype=torch.int32, device=dev, generator=gen)
        svh = (torch.randint(0, 2, (n,), device=dev, generator=gen).to(torch.float16) * 2 - 1)
        wt = torch.empty((n, k), dtype=torch.float16, device=dev)
        for M in (512, 4096):
            xh = torch.randn((M, k), device=dev, generator=gen).to(torch.float16)
            y = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
            yh = torch.empty((M, n), dtype=torch.float16, device=dev)

            def fused():
                kernels.gemm(xh, tr, k, n, K, 0, svh, torch.bfloat16, out=y)

            def decode_once():
                kernels.decode_wt(tr, k, n, K, 0, out=wt)
                kernels.gemm_wt(xh, wt, svh, out=y)

            def gemm_alone():
                kernels.gemm_wt(xh, wt, svh, out=y)

            def decode_once_cublas():
                kernels.decode_wt(tr, k, n, K, 0, out=wt)
                torch.matmul(xh, wt.t(), out=yh)
                kernels.had_svh(yh, svh, torch.bfloat16)

            res = {"M": M, "k": k, "n": n, "bits": K,
                   "default": "fused_tcgen05" if use_fused(M, n) else "decode_once_tcgen05"}
            for name, fn in (("fused_tcgen05", fused), ("decode_once_tcgen05", decode_once),
                             ("gemm_wt_alone", gemm_alone), ("decode_once_cublas", decode_once_cublas)):
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
            cases.append(res)
            del xh, y, yh
        del tr, wt
    torch.cuda.empty_cache()
    return {"peak_TFLOPs": tf_peak, "peak_kind": f"{peaks['kind']} bf16 burst (each call timed alone; fp16 has the "
                                                  "same rate)", "status": kernels.gemm_status(dev), "cases": cases}


# ------------------------------------------------------------------------------------------ CPU

def _cpu_lib():
    """The reference's decode source compiled for the host (oracle/_ref), else this repo's C port."""
    from oracle import oracle as O
    L = O.ref_lib()
    threads = os.cpu_count() or 1
    if L is not None:
        L.exl3_ref_set_threads(threads)
        return O, L, "reference", threads
    O.lib().exl3o_set_threads(threads)
    return O, None, "port", threads


def _cpu_gemv(O, L, t, k, n, K, xh, svh):
    if L is not None:
        y = np.empty((1, n), np.float32)
        L.exl3_ref_gemv(K, 0, O._ptr(O.trellis_u32(t)), k, n, O._ptr(xh.view(np.uint16)), 1,
                        O._ptr(svh.view(np.uint16)), O._ptr(y))
        return y
    return O.gemv_c(t, k, n, K, 0, xh, svh)


def cpu_decode_sample(budget_s: float = 10.0):
    """The reference's CPU path on a bounded sample of the config-5 decode step: every (k, bitrate) of
    the model's linears is timed on a 2048-column slice (decode + fp32 GEMV + rotation per call, all host
    threads) to get seconds per weight, plus one layer's attention over the 4096-token cache in numpy;
    tok/s = 1 / (sum over the model's 64 layers and the head of weights x seconds per weight +
    64 x attention)."""
    from omlx_exl3_b200.loader import draw_bits
    O, L, kind, threads = _cpu_lib()
    cfg = model_cfg(64)
    bits = draw_bits(64, seed=0, cfg=cfg)
    h, hd, ni = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    shapes = {"q_proj": (h, cfg.num_attention_heads * hd), "k_proj": (h, cfg.num_key_value_heads * hd),
              "v_proj": (h, cfg.num_key_value_heads * hd), "o_proj": (cfg.num_attention_heads * hd, h),
              "gate_proj": (h, ni), "up_proj": (h, ni), "down_proj": (ni, h)}
    need = {}                                  # (k, K) -> weights per token
    for lb in bits:
        for name, (k, n) in shapes.items():
            need[(k, lb[name])] = need.get((k, lb[name]), 0) + k * n
    vocab = ((cfg.vocab_size + 127) // 128) * 128
    need[(h, 8)] = need.get((h, 8), 0) + h * vocab
    rng = np.random.default_rng(0)
    per_key = max(0.2, budget_s * 0.8 / len(need))
    sec_per_weight, sample = {}, []
    nc = 2048
    for (k, K) in sorted(need):
        t = O.random_trellis(k, nc, K, 77 + K)
        xh = rng.standard_normal((1, k)).astype(np.float16)
        svh = np.where(rng.random(nc) < 0.5, -1, 1).astype(np.float16)
        _cpu_gemv(O, L, t, k, nc, K, xh, svh)
        calls, t0 = 0, time.perf_counter()
        while True:
            _cpu_gemv(O, L, t, k, nc, K, xh, svh)
            calls += 1
            if time.perf_counter() - t0 > per_key:
                break
        sec_per_weight[(k, K)] = (time.perf_counter() - t0) / calls / (k * nc)
        sample.append(f"{k}x{nc}@{K}bpw x{calls}")
    # one layer's attention (8 kv heads x 5 q heads, 4096 cached positions, fp32 numpy)
    kc = rng.standard_normal((cfg.num_key_value_heads, KV_LEN, hd)).astype(np.float32)
    vc = rng.standard_normal((cfg.num_key_value_heads, KV_LEN, hd)).astype(np.float32)
    q = rng.standard_normal((cfg.num_attention_heads, hd)).astype(np.float32)
    g = cfg.num_attention_heads // cfg.num_key_value_heads
    reps, t0 = 0, time.perf_counter()
    while True:
        for kv in range(cfg.num_key_value_heads):
            s = q[kv * g:(kv + 1) * g] @ kc[kv].T / np.sqrt(hd)
            p = np.exp(s - s.max(-1, keepdims=True))
            (p / p.sum(-1, keepdims=True)) @ vc[kv]
        reps += 1
        if time.perf_counter() - t0 > budget_s * 0.2:
            break
    attn_s = (time.perf_counter() - t0) / reps
    token_s = sum(w * sec_per_weight[key] for key, w in need.items()) + cfg.num_hidden_layers * attn_s
    return {"value": round(1.0 / token_s, 5), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"per-(k, bpw) GEMV seconds per weight from {', '.join(sample)}; numpy attention "
                      f"{attn_s * 1e3:.1f} ms/layer; extrapolated to the 64-layer model + 8-bpw head "
                      f"({token_s:.1f} s per token) on {threads} host threads"}


def cpu_config1(budget_s: float = 5.0):
    """BASELINE config 1 on the host: 4096 -> 4096 at 4 bpw, batch 1 (decode + fp32 GEMV + rotation)."""
    O, L, kind, threads = _cpu_lib()
    k = n = 4096
    K = 4
    rng = np.random.default_rng(1)
    t = O.random_trellis(k, n, K, 5)
    xh = rng.standard_normal((1, k)).astype(np.float16)
    svh = np.where(rng.random(n) < 0.5, -1, 1).astype(np.float16)
    _cpu_gemv(O, L, t, k, n, K, xh, svh)
    calls, t0 = 0, time.perf_counter()
    while True:
        _cpu_gemv(O, L, t, k, n, K, xh, svh)
        calls += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = (time.perf_counter() - t0) / calls
    b = gemv_bytes(k, [n], [K], 1)
    return {"GBps": round(b / dt / 1e9, 4), "us": round(dt * 1e6, 1), "cores": threads, "kind": kind,
            "sample": f"{calls} calls"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    budget = max(4.0, min(15.0, 90.0 / max(1, args.steps + 1)))
    for _ in range(min(args.warmup, 1)):
        cpu_decode_sample(budget_s=2.0)
    samples = [cpu_decode_sample(budget_s=budget) for _ in range(max(1, min(args.steps, 5)))]
    v = float(np.median([s["value"] for s in samples]))
    cpu = dict(samples[-1])
    cpu["value"] = v
    c1 = cpu_config1(budget_s=4.0)
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / v, 1) if v else None,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded uniform trellis, +-1 suh/svh, fp16 N(0,1) activations)",
        "config": {"workload": "BASELINE config 5: batch-1 decode of the random-init 64-layer 27B-class model, "
                               "4096-token KV cache; bounded CPU sample extrapolated to tok/s",
                   "note": "the reference's Metal path cannot run on this box; CPU = its decode source compiled by "
                           "oracle/build_ref.py + fp32 GEMV + FWHT, numpy attention"},
        "config1": {"workload": "BASELINE config 1: 4096->4096, 4 bpw, batch 1, 3inst", **c1},
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------------------------------ main

def run_ours(args, torch, dist, rank, world, dev):
    peaks = load_peaks()
    dec = run_decode(args, torch, dist, rank, world, dev, layers=args.decode_layers, rows=1, head=True,
                     gemv_roofline=(world == 1))
    extra = {}
    if not args.decode_only:
        extra["layer"] = run_decode(args, torch, dist, rank, world, dev, layers=1, rows=1, head=False)
        extra["verify"] = run_decode(args, torch, dist, rank, world, dev, layers=args.decode_layers, rows=4,
                                     head=True)
        if world > 1:
            extra["tp_parity"] = run_tp_parity(torch, dist, rank, world, dev)
        if world == 1:
            extra["gemv_sweep"] = run_sweep(args, torch, dev, peaks)
            extra["config1"] = run_config1(args, torch, dev, peaks)
            if not args.no_prefill:
                extra["prefill_gemm"] = run_prefill(args, torch, dev, peaks)
    if rank != 0:
        return None
    value = dec["tok_s"]
    gemv = dec.get("gemv")
    roof = {"bound": "hbm", "peak": peaks["hbm"], "unit": "GB/s", "peak_kind": peaks["kind"],
            "kernel": "exl3::gemv_kernel / gemv_seg_kernel (the step's GEMV launches replayed alone)"}
    if gemv:
        roof.update(achieved=gemv["achieved_GBps"], frac=round(gemv["achieved_GBps"] / peaks["hbm"], 4),
                    # DRAM (read + write) / algorithmic bytes of one ncu capture of the GEMV, per launch
                    traffic=int(gemv["bytes_per_launch"] * 1.004), traffic_unit="bytes per launch",
                    launches=gemv["launches"], us_per_launch=gemv["us_per_launch"])
    roof["step_GBps_per_gpu"] = dec["step_GBps_per_gpu"]
    roof["step_frac"] = round(dec["step_GBps_per_gpu"] / peaks["hbm"], 4)
    out = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": dec["steps"],
        "warmup": args.warmup, "ms_per_step": dec["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded uniform trellis, +-1 suh/svh, N(1,0.1) norms, N(0,1) embeddings and KV cache)",
        "accumulate": "fp32",
        "config": {"workload": f"BASELINE config 5: batch-1 decode, random-init {args.decode_layers}-layer 27B-class "
                               "model (hidden 5120, 40q/8kv x 128, SwiGLU 17408, vocab 151936, 8-bpw EXL3 head, "
                               "per-tensor 5..8 bpw averaging 6.0), 4096-token fp16 KV cache, CUDA-graph step",
                   "global_batch": 1, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2: each step streams all ~17 GB of weights"},
        "roofline": roof,
        "clocks": dec["clocks"],
        "gpu_launches": dec["launches_per_step"] * dec["steps"],
        "e2e": {"value": dec["e2e_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                "path": "DecodeRunner.step: token from pinned host memory, greedy next token back, every step"},
        "decode": {k: v for k, v in dec.items() if k not in ("clocks", "gemv")},
        **extra,
    }
    if world == 1 and not args.no_cpu_baseline and not args.decode_only:
        out["cpu_baseline"] = cpu_decode_sample(budget_s=10.0)
        if "config1" in out:
            c1 = cpu_config1(budget_s=3.0)
            out["config1"]["cpu_reference"] = {**c1, "same_config": True}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill GEMM measurement")
    ap.add_argument("--decode-layers", type=int, default=64)
    ap.add_argument("--decode-only", action="store_true", help="only the headline decode measurement")
    ap.add_argument("--tp-parity-only", action="store_true", help="only the tensor-parallel logit check")
    ap.add_argument("--prefill-only", action="store_true", help="only the config-3 prefill GEMM measurement")
    ap.add_argument("--timeline", action="store_true",
                    help="per-kernel critical-path breakdown of the decode step (--decode-layers layers)")
    ap.add_argument("--sweep-case", default=None,
                    help="k,n,K,rows: time one GEMV configuration alone and exit (small ncu captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if args.sweep_case:
            global SWEEP_SHAPES, SWEEP_BITS, SWEEP_ROWS
            k, n, K, rows = (int(v) for v in args.sweep_case.split(","))
            SWEEP_SHAPES, SWEEP_BITS, SWEEP_ROWS = [(k, n)], [K], [rows]
            print(json.dumps({"sweep_case": run_sweep(args, torch, dev, load_peaks())}), flush=True)
            return
        if args.prefill_only:
            print(json.dumps({"prefill_gemm": run_prefill(args, torch, dev, load_peaks())}), flush=True)
            return
        if args.timeline:
            res = run_timeline(args, torch, dist, rank, world, dev, layers=args.decode_layers)
            if res is not None:
                print(json.dumps(res), flush=True)
            return
        if args.tp_parity_only:
            res = run_tp_parity(torch, dist, rank, world, dev)
            if rank == 0:
                print(json.dumps({"tp_parity": res, "n_gpus": world}), flush=True)
            return
        out = run_ours(args, torch, dist, rank, world, dev)
        if out is not None:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
