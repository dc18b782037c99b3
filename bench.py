#!/usr/bin/env python3
"""Benchmark of the MatMulNBits int4 hot path on B200.

Headline (one JSON line on rank 0): MatMulNBits int4 decode GEMV HBM
throughput in GB/s, BASELINE config 3 at M=1 (K=1024, N=3072, block 32,
packed uint4 zero points). One step = one decode token through a stack of
`--layers` x `--passes` config-3 layers (256 distinct weight sets, each reused
every 516 MB of weight traffic, so the stream exceeds the 126 MB L2 and every
timed byte comes from HBM), launched back to back (captured in a CUDA graph;
each kernel prefetches its weights under programmatic dependent launch). The
same line carries the M=512 prefill TFLOP/s and M=8 decode GB/s (same config),
the end-to-end number through the host-buffer C-ABI call, the roofline of the
dominant kernel, the CPU baseline (the oracle port of the reference's Dart
kernel on the host cores) and SM clocks sampled during the timed region.

N > 1 runs under torchrun: every rank drives its own GPU with its own weight
stack (replicas: config 3 is a single op and shards no data; weak scaling),
times on the device with CUDA events, and the slowest rank's time is used.
`--impl reference` times the reference's CPU implementation (the oracle
restatement; the Dart VM is not available) on the same metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_DIM, N_DIM, BLOCK = 1024, 3072, 32
NB = K_DIM // BLOCK
W_BYTES = N_DIM * K_DIM // 2 + N_DIM * NB * 4 + N_DIM * ((NB + 1) // 2)  # 2,015,232
METRIC = "MatMulNBits int4 decode GEMV HBM GB/s"


def launch_bytes(m):
    return W_BYTES + m * K_DIM * 4 + m * N_DIM * 4


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def committed_traffic(name):
    """dram read+write bytes per launch from a committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


def make_weights(rng, n_sets):
    """Seeded config-3 weights: nibbles uniform [0,15], scales |N(0,.02)|+1e-3,
    packed uint4 zero points uniform [0,15]."""
    out = []
    for _ in range(n_sets):
        bq = rng.integers(0, 256, (N_DIM, NB, BLOCK // 2), dtype=np.uint8)
        sc = (np.abs(rng.normal(0, 0.02, (N_DIM, NB))) + 1e-3).astype(np.float32)
        zp = rng.integers(0, 256, (N_DIM, (NB + 1) // 2), dtype=np.uint8)
        out.append((bq, sc, zp))
    return out


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# reference arm: the CPU implementation of the path
# ---------------------------------------------------------------------------

def cpu_decode_gbs(steps, warmup, layers_per_step, threads, seed=0):
    import oracle
    rng = np.random.default_rng(seed)
    ws = make_weights(rng, 4)
    a = rng.standard_normal((1, K_DIM)).astype(np.float32)
    for i in range(warmup * layers_per_step):
        bq, sc, zp = ws[i % len(ws)]
        oracle.matmul_nbits(a, bq, sc, zp, K_DIM, N_DIM, BLOCK, nthreads=threads)
    t0 = time.perf_counter()
    for i in range(steps * layers_per_step):
        bq, sc, zp = ws[i % len(ws)]
        oracle.matmul_nbits(a, bq, sc, zp, K_DIM, N_DIM, BLOCK, nthreads=threads)
    dt = time.perf_counter() - t0
    return steps * layers_per_step * launch_bytes(1) / dt / 1e9, dt


def _best_time(fn, reps):
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def cpu_baselines(threads, seed=0):
    """The oracle port (C restatement of the reference Dart kernels, compiled
    -O2 -ffp-contract=off; not the Dart VM, which is not installed) timed per
    BASELINE config on the host cores: 1 thread, and `threads` threads
    column-splitting each MatMul the way the reference's GemmPool splits
    float-initializer MatMuls (lib/src/parallel_pool.dart:236-260; the
    reference itself pools only those, not MatMulInteger / MatMulNBits,
    lib/src/onnx_graph.dart:856-872). Best of a few runs after a warm-up run.
    Chains are truncated as stated in each entry."""
    import platform

    import oracle
    from oracle import chains
    from onnx_runtime_dart_b200.bert import BertConfig
    from onnx_runtime_dart_b200.decoder import DecoderConfig

    rng = np.random.default_rng(seed)
    out = {"what": "oracle port of the reference Dart kernels (C, -O2 -ffp-contract=off), not the Dart VM",
           "threads": threads, "cpu": platform.processor() or platform.machine()}
    try:
        with open("/proc/cpuinfo") as f:
            names = [ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")]
        if names:
            out["cpu"] = names[0]
    except OSError:
        pass

    def both(fn, reps=3):
        fn(1)
        return _best_time(lambda: fn(1), reps), _best_time(lambda: fn(threads), reps)

    a = rng.standard_normal((128, 384)).astype(np.float32)
    b = (rng.standard_normal((384, 1536)) / np.sqrt(384)).astype(np.float32)
    t1, tn = both(lambda th: oracle.matmul(a, b, nthreads=th), 5)
    fl = 2 * 128 * 384 * 1536
    out["config1_matmul_f32_gflops"] = {"1_thread": round(fl / t1 / 1e9, 3), f"{threads}_threads": round(fl / tn / 1e9, 3)}
    bi = rng.integers(-127, 128, (1024, 3072)).astype(np.int8)
    bz = rng.integers(-4, 5, 3072).astype(np.int8)
    az = np.array(128, np.uint8)
    c2 = {}
    for m in (1, 64, 512):
        ai = rng.integers(0, 256, (m, 1024)).astype(np.uint8)
        t1, tn = both(lambda th: oracle.matmul_integer(ai, bi, az, bz, nthreads=th), 3 if m < 512 else 2)
        ops = 2 * m * 1024 * 3072
        c2[f"m{m}"] = {"1_thread_gops": round(ops / t1 / 1e9, 3), f"{threads}_threads_gops": round(ops / tn / 1e9, 3),
                       "1_thread_ms": round(t1 * 1e3, 3)}
    out["config2_matmulinteger"] = c2
    bq = rng.integers(0, 256, (N_DIM, NB, BLOCK // 2), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, (N_DIM, NB))) + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, (N_DIM, (NB + 1) // 2), dtype=np.uint8)
    c3 = {}
    for m in (1, 8, 512):
        x = rng.standard_normal((m, K_DIM)).astype(np.float32)
        t1, tn = both(lambda th: oracle.matmul_nbits(x, bq, sc, zp, K_DIM, N_DIM, BLOCK, nthreads=th), 3 if m < 512 else 2)
        e = {"1_thread_ms": round(t1 * 1e3, 3), f"{threads}_threads_ms": round(tn * 1e3, 3)}
        if m < 512:
            e["1_thread_gbs"] = round(launch_bytes(m) / t1 / 1e9, 3)
            e[f"{threads}_threads_gbs"] = round(launch_bytes(m) / tn / 1e9, 3)
        else:
            fl = 2 * m * K_DIM * N_DIM
            e["1_thread_gflops"] = round(fl / t1 / 1e9, 3)
            e[f"{threads}_threads_gflops"] = round(fl / tn / 1e9, 3)
        c3[f"m{m}"] = e
    out["config3_matmulnbits"] = c3

    # config 4: one sequence of 128 tokens (of the 32 x 128 batch); all 12
    # layers on `threads` threads, the first 2 layers on 1 thread.
    bc = BertConfig.base()
    bh = chains.bert_host(bc, seed)
    ids = rng.integers(0, bc.vocab, (1, 128)).astype(np.int64)
    mask = np.ones((1, 128), np.int64)
    tn = _best_time(lambda: chains.bert_forward(bc, bh, ids, mask, nthreads=threads), 1)
    bc2 = BertConfig.base()
    bc2.layers = 1
    t1 = _best_time(lambda: chains.bert_forward(bc2, bh, ids, mask, nthreads=1), 1)
    out["config4_bert"] = {"sample": "1 sequence x 128 tokens; 12 layers on all threads, 1 layer on 1 thread",
                           f"{threads}_threads_tokens_per_s": round(128 / tn, 2),
                           "1_thread_ms_per_layer": round(t1 * 1e3, 2),
                           "1_thread_tokens_per_s_12_layers_derived": round(128 / (t1 * 12), 2)}
    del bh

    # config 5: one sequence, 32-token prefill then 2 greedy decode steps;
    # all 28 layers on `threads` threads, 2 layers on 1 thread (the lm_head
    # included in both).
    dc = DecoderConfig.qwen3_0_6b()
    dh = chains.decoder_host(dc, seed)
    prompt = rng.integers(0, dc.vocab, (1, 32)).astype(np.int64)

    def run_dec(cfg, th):
        t0 = time.perf_counter()
        lg, past = chains.decoder_forward(cfg, dh, 40, prompt, None, strict=True, nthreads=th)
        t1_ = time.perf_counter()
        tok = np.argmax(lg, axis=-1).reshape(1, 1)
        for _ in range(2):
            lg, past = chains.decoder_forward(cfg, dh, 40, tok, past, strict=True, nthreads=th)
            tok = np.argmax(lg, axis=-1).reshape(1, 1)
        return t1_ - t0, time.perf_counter() - t1_

    pn, dn = run_dec(dc, threads)
    dc2 = DecoderConfig.qwen3_0_6b()
    dc2.layers = 2
    p1, d1 = run_dec(dc2, 1)
    out["config5_decoder"] = {"sample": "1 sequence, 32-token prefill + 2 greedy decode steps; 28 layers on all "
                                        "threads, 2 layers on 1 thread (lm_head included in both)",
                              f"{threads}_threads_prefill_tokens_per_s": round(32 / pn, 2),
                              f"{threads}_threads_decode_tokens_per_s": round(2 / dn, 3),
                              "1_thread_2_layers_prefill_ms": round(p1 * 1e3, 1),
                              "1_thread_2_layers_decode_ms_per_step": round(d1 * 1e3 / 2, 1)}
    del dh
    return out


def run_reference(args, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    layers = 8
    gbs, dt = cpu_decode_gbs(args.steps, args.warmup, layers, threads)
    sample = (f"oracle restatement of opMatMulNBits m==1 (double accumulation, "
              f"onnx_qlinear_ops.dart:194-205), {layers} config-3 layers per step, column split over "
              f"{threads} threads (parallel_pool.dart:236-239)")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64 accumulate (reference m==1 path)", "data": "synthetic (seeded)",
        "config": {"workload": "MatMulNBits decode, BASELINE config 3 M=1 (K=1024 N=3072 block 32 packed zp)",
                   "layers_per_step": layers, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# BASELINE configs 1 and 2 (single ops, device-resident operands)
# ---------------------------------------------------------------------------

def _time_calls(torch, stream, fn, steps, warmup):
    for _ in range(max(3, warmup)):
        fn()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    stream.synchronize()
    return e0.elapsed_time(e1) / steps  # ms per call


def _time_graph(torch, ctx, stream, calls, steps, warmup):
    """Device time per call of `calls` (a list of zero-argument launchers)
    captured back to back in one CUDA graph, replayed `steps` times."""
    for fn in calls:  # eager warm-up outside capture (kernel attributes, scratch growth)
        fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        for fn in calls:
            fn()
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            g.replay()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            g.replay()
        e1.record(stream)
    stream.synchronize()
    del g
    return e0.elapsed_time(e1) / (steps * len(calls))


def other_configs(ctx, lib, N, stream, dev, steps, warmup):
    """Config 1: fp32 MatMul A[128,384] x B[384,1536] (B prepacked), EXACT and
    FAST modes. Config 2: MatMulInteger u8[M,1024] x i8[1024,3072], aZp=128,
    per-column bZp in [-4,4], M in {1, 64, 512}. Device-resident inputs.
    `us_per_call`: eager calls through the C ABI, back to back on one stream
    (host overhead included, one weight set). `graph_us_per_call`: the same
    calls over SETS distinct weight sets and outputs (more than L2 holds)
    captured in one CUDA graph: device time per op."""
    import torch
    SETS = 64
    rng = np.random.default_rng(0)
    out = []
    a = rng.standard_normal((128, 384)).astype(np.float32)
    da = ctx.upload(a)
    wbs = [ctx.prepack_f32((rng.standard_normal((384, 1536)) / np.sqrt(384)).astype(np.float32)) for _ in range(SETS)]
    dys = [ctx.empty((128, 1536)) for _ in range(SETS)]

    def f32_call(i, mode):
        def call():
            h = ctypes.c_void_p(dys[i].handle.value)
            N.check(lib.b2m_matmul_f32(ctx.handle, da.handle, None, wbs[i].handle, mode, ctypes.byref(h)))
        return call
    for mode, name in ((N.MODE_EXACT, "exact"), (N.MODE_FAST, "fast")):
        ms = _time_calls(torch, stream, f32_call(0, mode), steps * 10, warmup)
        gms = _time_graph(torch, ctx, stream, [f32_call(i, mode) for i in range(SETS)], steps, warmup)
        flop = 2 * 128 * 384 * 1536
        out.append({"case": f"config1_matmul_f32_{name}", "us_per_call": ms * 1e3, "graph_us_per_call": gms * 1e3,
                    "TFLOPs": flop / (gms / 1e3) / 1e12,
                    "GBps": 4 * (128 * 384 + 384 * 1536 + 128 * 1536) / (gms / 1e3) / 1e9})
    for w in wbs:
        w.free()
    wis = [ctx.prepack_i8(rng.integers(-127, 128, (1024, 3072)).astype(np.int8)) for _ in range(SETS)]
    az = ctx.upload(np.array(128, np.uint8))
    bz = ctx.upload(rng.integers(-4, 5, (3072,)).astype(np.int8))
    for m in (1, 64, 512):
        ai = ctx.upload(rng.integers(0, 256, (m, 1024)).astype(np.uint8))
        yis = [ctx.empty((m, 3072), np.int32) for _ in range(SETS)]

        def i8_call(i):
            def call():
                h = ctypes.c_void_p(yis[i].handle.value)
                N.check(lib.b2m_matmul_integer(ctx.handle, ai.handle, None, wis[i].handle, az.handle, bz.handle,
                                               ctypes.byref(h)))
            return call
        ms = _time_calls(torch, stream, i8_call(0), steps * 10, warmup)
        gms = _time_graph(torch, ctx, stream, [i8_call(i) for i in range(SETS)], steps, warmup)
        ops = 2 * m * 1024 * 3072
        by = m * 1024 + 1024 * 3072 + 3072 + m * 3072 * 4
        out.append({"case": f"config2_matmulinteger_m{m}", "us_per_call": ms * 1e3, "graph_us_per_call": gms * 1e3,
                    "TOPs": ops / (gms / 1e3) / 1e12, "GBps": by / (gms / 1e3) / 1e9})
    for w in wis:
        w.free()
    return out


def run_decoder(ctx, torch, stream, global_batch, prefill_len=512, steps=128, layers=None, seed=0, world=1, rank=0,
                fused=True, mode=None):
    """Qwen3-0.6B-shaped int4 decoder (random weights,
    replicated on every rank). This rank runs its slice of the
    `global_batch` sequences (a seeded global prompt of `prefill_len` tokens
    each), then `steps` greedy decode steps replayed as one CUDA graph per
    step. Device time (CUDA events)."""
    from onnx_runtime_dart_b200 import sharding
    from onnx_runtime_dart_b200.decoder import DecoderConfig, Int4Decoder

    cfg = DecoderConfig.qwen3_0_6b()
    if layers:
        cfg.layers = layers
    rng = np.random.default_rng(seed + 1)
    prompt_all = rng.integers(0, cfg.vocab, (global_batch, prefill_len)).astype(np.int64)
    prompt = sharding.local_slice(prompt_all, world, rank)
    batch = len(prompt)
    from onnx_runtime_dart_b200 import _native as N

    dec = Int4Decoder(ctx, cfg, batch=batch, cap=prefill_len + steps + 8, max_prefill=prefill_len, seed=seed,
                      fused=fused, mode=N.MODE_FAST if mode is None else mode)
    with torch.cuda.stream(stream):
        dec.prefill(prompt)  # warm-up (kernel attributes, scratch growth)
        dec.decode(2)        # captures the decode graph
        stream.synchronize()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        dec.prefill(prompt)
        e1.record(stream)
        gen = dec.decode(steps)
        e2.record(stream)
        stream.synchronize()
    ms_p, ms_d = e0.elapsed_time(e1), e1.elapsed_time(e2)
    ok = bool(((gen >= 0) & (gen < cfg.vocab)).all().item())
    out = {"batch_per_gpu": batch, "prefill_len": prefill_len, "decode_steps": steps, "layers": cfg.layers,
           "projections": ("fused q/k/v and gate/up (SwiGLU in the gate/up epilogue; q/k head norms, rotary and "
                           "cache append in the attention)" if fused
                           else "separate (the exported graph's seven per layer)"),
           "prefill_ms": round(ms_p, 3), "decode_ms": round(ms_d, 3),
           "prefill_tokens_per_s": round(batch * prefill_len / (ms_p / 1e3), 1),
           "decode_tokens_per_s": round(batch * steps / (ms_d / 1e3), 1),
           "decode_ms_per_step": round(ms_d / steps, 4), "tokens_valid": ok}
    del dec
    torch.cuda.empty_cache()
    return out


def run_bert(ctx, torch, stream, global_batch, seq=128, steps=10, warmup=3, layers=None, seed=0, exact=False,
             world=1, rank=0):
    """BERT-base-shaped fp32 encoder (random weights,
    replicated on every rank) over this rank's slice of `global_batch`
    sequences of `seq` tokens, all-ones attention mask. Device time of one
    graph-replayed forward (CUDA events, mean over `steps`), and the same
    forward end to end: ids from pinned host memory in, the last hidden state
    back to pinned host memory."""
    from onnx_runtime_dart_b200 import _native as N
    from onnx_runtime_dart_b200 import sharding
    from onnx_runtime_dart_b200.bert import BertConfig, BertEncoder

    cfg = BertConfig.base()
    if layers:
        cfg.layers = layers
    rng = np.random.default_rng(seed + 1)
    ids = sharding.local_slice(rng.integers(0, cfg.vocab, (global_batch, seq)).astype(np.int64), world, rank)
    batch = len(ids)
    enc = BertEncoder(ctx, cfg, batch, seq, seed=seed, mode=N.MODE_EXACT if exact else N.MODE_FAST)
    ids_pin = torch.from_numpy(ids.reshape(-1)).pin_memory()
    out_pin = torch.empty((batch * seq, cfg.hidden), dtype=torch.float32).pin_memory()
    with torch.cuda.stream(stream):
        enc.set_attention_mask(np.ones((batch, seq)))
        enc.ids.copy_(ids_pin, non_blocking=True)
        for _ in range(max(1, warmup)):
            enc.forward_device(True)
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            enc.forward_device(True)
        e1.record(stream)
        stream.synchronize()
        ms_dev = e0.elapsed_time(e1) / steps
        e0.record(stream)
        for _ in range(steps):
            enc.ids.copy_(ids_pin, non_blocking=True)
            enc.forward_device(True)
            out_pin.copy_(enc.x, non_blocking=True)
        e1.record(stream)
        stream.synchronize()
        ms_e2e = e0.elapsed_time(e1) / steps
    finite = bool(np.isfinite(out_pin.numpy()).all())
    flops = cfg.flops_per_token(seq) * batch * seq
    out = {"batch_per_gpu": batch, "seq": seq, "layers": cfg.layers, "mode": "exact" if exact else "fast-bf16x3",
           "forward_ms": round(ms_dev, 4), "e2e_forward_ms": round(ms_e2e, 4),
           "flop_per_forward": flops, "tflops": round(flops / (ms_dev / 1e3) / 1e12, 2),
           "h2d_bytes": int(ids.nbytes), "d2h_bytes": int(out_pin.numel() * 4), "finite": finite}
    del enc
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def conv_configs(ctx, lib, N, stream, steps, warmup):
    """Convolutions through the GEMM cores on a ResNet-style 3x3 layer
    (x [32, 64, 56, 56], w [64, 64, 3, 3], pads 1, bias): Conv FAST (bf16
    split planes on tcgen05) and EXACT (fp32, the reference's k order), and
    QLinearConv u8 x i8 -> u8. Four distinct inputs / weights / outputs per
    CUDA graph (the FAST im2col panel, 231 MB per call, exceeds L2).
    Device time per call; FLOP = 2 * n * P * M * K (useful work)."""
    import torch
    SETS = 4
    n, c, hw, m, k = 32, 64, 56, 64, 3
    rng = np.random.default_rng(2)
    xs = [ctx.upload(rng.standard_normal((n, c, hw, hw)).astype(np.float32)) for _ in range(SETS)]
    ws = [ctx.prepack_conv((rng.standard_normal((m, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32))
          for _ in range(SETS)]
    bs = [ctx.upload(rng.standard_normal(m).astype(np.float32)) for _ in range(SETS)]
    ys = [ctx.empty((n, m, hw, hw)) for _ in range(SETS)]
    flop = 2 * n * hw * hw * m * c * k * k
    ks = np.array([k, k], np.int64)
    pads = np.array([1, 1, 1, 1], np.int64)
    vp = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    out = {"shape": f"x[{n},{c},{hw},{hw}] w[{m},{c},{k},{k}] pads 1"}

    def f32_call(i, mode):
        def call():
            h = ctypes.c_void_p(ys[i].handle.value)
            N.check(lib.b2m_conv_f32(ctx.handle, xs[i].handle, ws[i].handle, bs[i].handle, vp(ks), None, vp(pads),
                                     None, 1, 0, mode, ctypes.byref(h)))
        return call
    for mode, name in ((N.MODE_FAST, "fast"), (N.MODE_EXACT, "exact")):
        gms = _time_graph(torch, ctx, stream, [f32_call(i, mode) for i in range(SETS)], steps, warmup)
        out[f"conv_{name}_us"] = round(gms * 1e3, 2)
        out[f"conv_{name}_tflops"] = round(flop / (gms / 1e3) / 1e12, 2)
    xq = [ctx.upload(rng.integers(0, 256, (n, c, hw, hw)).astype(np.uint8)) for _ in range(SETS)]
    wq = [ctx.prepack_conv(rng.integers(-127, 128, (m, c, k, k)).astype(np.int8)) for _ in range(SETS)]
    xz = ctx.upload(np.array(128, np.uint8))
    wz = ctx.upload(np.array(0, np.int8))
    bq = ctx.upload(rng.integers(-1000, 1000, m).astype(np.int32))
    wscale = ctx.upload(np.full(m, 0.004, np.float32))
    yq = [ctx.empty((n, m, hw, hw), np.uint8) for _ in range(SETS)]

    def q_call(i):
        def call():
            h = ctypes.c_void_p(yq[i].handle.value)
            N.check(lib.b2m_qlinear_conv(ctx.handle, xq[i].handle, 0.02, xz.handle, wq[i].handle, wscale.handle,
                                         wz.handle, 0.5, 128, bq.handle, vp(ks), None, vp(pads), None, 1, 0, 255,
                                         ctypes.byref(h)))
        return call
    gms = _time_graph(torch, ctx, stream, [q_call(i) for i in range(SETS)], steps, warmup)
    out["qlinearconv_us"] = round(gms * 1e3, 2)
    out["qlinearconv_tops"] = round(flop / (gms / 1e3) / 1e12, 2)
    for w in ws + wq:
        w.free()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=256, help="distinct weight sets (516 MB for 256)")
    ap.add_argument("--passes", type=int, default=64,
                    help="passes over the weight sets per decode step (step = layers x passes launches)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-weight-links", action="store_true",
                    help="do not declare each weight set's successor (no cross-call L2 prefetch)")
    ap.add_argument("--case", default="all",
                    choices=["all", "decode1", "decode8", "prefill", "ops", "decoder", "bert", "conv", "cpu"],
                    help="run one phase only (for profiler captures); prints its device time. "
                         "`ops` times BASELINE configs 1 and 2 (fp32 MatMul, MatMulInteger); `conv` the "
                         "convolutions through the GEMM cores")
    ap.add_argument("--dec-layers", type=int, default=None, help="decoder case: layers (default 28)")
    ap.add_argument("--dec-steps", type=int, default=128, help="decoder case: greedy decode steps")
    ap.add_argument("--dec-unfused", action="store_true",
                    help="decoder case: separate q/k/v and gate/up MatMulNBits (the exported graph's projections)")
    ap.add_argument("--dec-mode", default="fast", choices=["fast", "precise", "exact"],
                    help="decoder case: MatMulNBits numerics mode")
    ap.add_argument("--dec-batch", type=int, default=None,
                    help="decoder case: sequences of the whole job, split over the ranks (default 64)")
    ap.add_argument("--bert-layers", type=int, default=None, help="bert case: layers (default 12)")
    ap.add_argument("--bert-exact", action="store_true", help="bert case: fp32-exact MatMuls instead of the FAST bf16-split tensor-core path")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank)
        return

    if args.case == "cpu":
        if rank == 0:
            print(json.dumps({"case": "cpu", **cpu_baselines(os.cpu_count() or 1)}), flush=True)
        return

    import torch
    import torch.distributed as dist

    import onnx_runtime_dart_b200 as b2m
    from onnx_runtime_dart_b200 import _native as N
    from onnx_runtime_dart_b200 import sharding

    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = b2m.Context(local)
    lib = ctx.lib
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        return sharding.max_over_ranks(x, dist if world > 1 else None, dev)

    if args.case == "bert":
        r = run_bert(ctx, torch, stream, 32, layers=args.bert_layers, exact=args.bert_exact, world=world, rank=rank,
                     steps=args.steps, warmup=args.warmup)
        t_f = max_over_ranks(r["forward_ms"])
        t_e = max_over_ranks(r["e2e_forward_ms"])
        if rank == 0:
            tok = 32 * r["seq"]  # the global batch, split over the ranks
            r["tokens_per_s_all_gpus"] = round(tok / (t_f / 1e3), 1)
            r["e2e_tokens_per_s_all_gpus"] = round(tok / (t_e / 1e3), 1)
            print(json.dumps({"case": "bert", **r}), flush=True)
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        return

    if args.case == "decoder":
        r = run_decoder(ctx, torch, stream, args.dec_batch or 64, steps=args.dec_steps, world=world, rank=rank,
                        layers=args.dec_layers, fused=not args.dec_unfused,
                        mode={"fast": N.MODE_FAST, "precise": N.MODE_PRECISE, "exact": N.MODE_EXACT}[args.dec_mode])
        t_p = max_over_ranks(r["prefill_ms"])
        t_d = max_over_ranks(r["decode_ms"])
        if rank == 0:
            gb = args.dec_batch or 64
            r["prefill_tokens_per_s_all_gpus"] = round(gb * r["prefill_len"] / (t_p / 1e3), 1)
            r["decode_tokens_per_s_all_gpus"] = round(gb * r["decode_steps"] / (t_d / 1e3), 1)
            print(json.dumps({"case": "decoder", **r}), flush=True)
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        return

    if args.case == "conv":
        r = conv_configs(ctx, lib, N, stream, args.steps, args.warmup)
        if rank == 0:
            print(json.dumps({"case": "conv", **r}), flush=True)
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        return

    rng = np.random.default_rng(1234 + rank)
    R = args.layers
    ws = make_weights(rng, R)
    packed = [ctx.prepack_nbits(bq, sc, zp, K_DIM, N_DIM, 4, BLOCK) for bq, sc, zp in ws]
    # The stack's call order, declared as a session would at load time: each
    # call's kernels prefetch the next call's weights into L2.
    if not args.no_weight_links:
        for i, w in enumerate(packed):
            w.set_next(packed[(i + 1) % R])

    def run_graph(m, layers, steps, warmup, passes=1):
        a = torch.randn((m, K_DIM), device=dev, dtype=torch.float32)
        ys = [torch.empty((m, N_DIM), device=dev, dtype=torch.float32) for _ in range(layers)]
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(layers):  # eager warm-up (kernel attributes set outside capture)
                N.check(lib.b2m_matmul_nbits_dev(ctx.handle, ctypes.c_void_p(a.data_ptr()), m, packed[i].handle,
                                                 None, N.MODE_FAST, ctypes.c_void_p(ys[i].data_ptr())))
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            ctx.set_stream(torch.cuda.current_stream().cuda_stream)
            for _ in range(passes):
                for i in range(layers):
                    N.check(lib.b2m_matmul_nbits_dev(ctx.handle, ctypes.c_void_p(a.data_ptr()), m, packed[i].handle,
                                                     None, N.MODE_FAST, ctypes.c_void_p(ys[i].data_ptr())))
        ctx.set_stream(stream.cuda_stream)
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                g.replay()
        stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.3)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                g.replay()
            e1.record(stream)
        stream.synchronize()
        clocks = sampler.stop()
        barrier()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1))
        del g
        return ms, clocks

    hbm_peak, tc_peak, peak_src = peaks()

    if args.case == "ops":
        for line in other_configs(ctx, lib, N, stream, dev, args.steps, args.warmup):
            if rank == 0:
                print(json.dumps(line), flush=True)
        ctx.close()
        return

    if args.case != "all":
        m = {"decode1": 1, "decode8": 8, "prefill": 512}[args.case]
        ms_c, clk_c = run_graph(m, R, args.steps, args.warmup)
        if rank == 0:
            print(json.dumps({"case": args.case, "M": m, "layers": R, "steps": args.steps, "clocks": clk_c,
                              "us_per_launch": ms_c * 1e3 / (args.steps * R),
                              "GBps": args.steps * R * launch_bytes(m) / (ms_c / 1e3) / 1e9,
                              "TFLOPs": args.steps * R * 2 * m * K_DIM * N_DIM / (ms_c / 1e3) / 1e12}), flush=True)
        for w in packed:
            w.free()
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        return

    # Headline: M=1 decode; one step = `passes` passes over the R weight sets.
    P = args.passes
    ms, clocks = run_graph(1, R, args.steps, max(3, args.warmup), passes=P)
    per_launch_s = ms / 1e3 / (args.steps * R * P)
    value = world * args.steps * R * P * launch_bytes(1) / (ms / 1e3) / 1e9
    achieved = launch_bytes(1) / per_launch_s / 1e9

    # M=8 decode (same rotation) and M=512 prefill (compute-bound).
    ms8, _ = run_graph(8, R, max(1, args.steps // 2), 3)
    gbs8 = args.steps // 2 * R * launch_bytes(8) / (ms8 / 1e3) / 1e9 if args.steps // 2 else None
    Rp = R  # 256 distinct weight sets: the prefill weights do not stay in L2 either
    msp, _ = run_graph(512, Rp, max(1, args.steps // 4), 3)
    tflops_p = max(1, args.steps // 4) * Rp * 2 * 512 * K_DIM * N_DIM / (msp / 1e3) / 1e12

    # BASELINE configs 1 and 2 (fp32 MatMul, int8 MatMulInteger): device time
    # per op over 64 weight sets in a CUDA graph.
    ops_lines = other_configs(ctx, lib, N, stream, dev, max(1, args.steps // 4), 3)
    conv_line = conv_configs(ctx, lib, N, stream, max(1, args.steps // 4), 3)

    # the int4 decoder chain, sequences sharded over ranks.
    dec = run_decoder(ctx, torch, stream, 64, world=world, rank=rank)
    dec_tp = max_over_ranks(dec["prefill_ms"])
    dec_td = max_over_ranks(dec["decode_ms"])
    dec_line = {"prefill_tokens_per_s": round(64 * dec["prefill_len"] / (dec_tp / 1e3), 1),
                "decode_tokens_per_s": round(64 * dec["decode_steps"] / (dec_td / 1e3), 1),
                "sequences": 64, "prefill_len": dec["prefill_len"],
                "decode_steps": dec["decode_steps"], "decode_ms_per_step": dec["decode_ms_per_step"],
                "mode": "FAST", "projections": dec["projections"], "tokens_valid": dec["tokens_valid"]}
    # The same decoder with the exported graph's separate projections, and in
    # PRECISE mode (the chain-parity mode), fused.
    for tag, kw in (("unfused_fast", dict(fused=False)), ("precise", dict(mode=N.MODE_PRECISE))):
        d2 = run_decoder(ctx, torch, stream, 64, world=world, rank=rank, **kw)
        tp2, td2 = max_over_ranks(d2["prefill_ms"]), max_over_ranks(d2["decode_ms"])
        dec_line[tag] = {"prefill_tokens_per_s": round(64 * d2["prefill_len"] / (tp2 / 1e3), 1),
                         "decode_tokens_per_s": round(64 * d2["decode_steps"] / (td2 / 1e3), 1),
                         "decode_ms_per_step": d2["decode_ms_per_step"], "projections": d2["projections"]}

    # the BERT-base fp32 chain, sequences sharded over ranks.
    bert = run_bert(ctx, torch, stream, 32, steps=5, warmup=3, world=world, rank=rank)
    bert_tf = max_over_ranks(bert["forward_ms"])
    bert_te = max_over_ranks(bert["e2e_forward_ms"])
    bert_tok = 32 * bert["seq"]
    bert_line = {"tokens_per_s": round(bert_tok / (bert_tf / 1e3), 1),
                 "e2e_tokens_per_s": round(bert_tok / (bert_te / 1e3), 1),
                 "forward_ms": bert["forward_ms"], "tflops_per_gpu": bert["tflops"],
                 "sequences": 32, "seq": bert["seq"], "mode": bert["mode"],
                 "finite": bert["finite"]}

    # End to end through the host-buffer C-ABI call (pinned host memory).
    e2e_layers = min(R, 64)
    a_h = torch.randn((1, K_DIM), dtype=torch.float32).pin_memory()
    y_h = torch.empty((1, N_DIM), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, args.steps // 2)
    for i in range(e2e_layers):
        N.check(lib.b2m_matmul_nbits_host(ctx.handle, ctypes.c_void_p(a_h.data_ptr()), 1, packed[i].handle, None,
                                          N.MODE_FAST, ctypes.c_void_p(y_h.data_ptr())))
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        for i in range(e2e_layers):
            N.check(lib.b2m_matmul_nbits_host(ctx.handle, ctypes.c_void_p(a_h.data_ptr()), 1, packed[i].handle,
                                              None, N.MODE_FAST, ctypes.c_void_p(y_h.data_ptr())))
    e1.record(stream)
    stream.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * e2e_steps * e2e_layers * launch_bytes(1) / (e2e_ms / 1e3) / 1e9

    # CPU baseline (rank 0 only, bounded sample of the same workload).
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        # size the sample to ~15 s of CPU work from a short probe
        probe_gbs, _ = cpu_decode_gbs(1, 1, 16, threads)
        layers = max(8, int(15.0 * probe_gbs * 1e9 / launch_bytes(1)))
        gbs_c, dt_c = cpu_decode_gbs(1, 0, layers, threads)
        cpu = {"value": round(gbs_c, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"oracle restatement of opMatMulNBits m==1 (double accumulation), {layers} config-3 "
                         f"layers ({dt_c:.1f} s), column split over {threads} threads"}

    cpu_all = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu_all = cpu_baselines(os.cpu_count() or 1)

    traffic = committed_traffic("nbits_decode_m1_k1024_n3072.md")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 (int4 weights exact in f16, f32 activations "
        "split f16 hi+lo, fp32 accumulate)", "data": "synthetic (seeded numpy default_rng)",
        "config": {"workload": "MatMulNBits int4 decode GEMV, BASELINE config 3 M=1 (K=1024 N=3072 block 32 "
                               "packed uint4 zp)", "M": 1, "K": K_DIM, "N": N_DIM, "block_size": BLOCK,
                   "layers_per_step": R * P, "distinct_weight_sets": R, "global_batch": world,
                   "parallelism": f"replicas x{world}",
                   "l2": f"weights rotated over {R * W_BYTES / 1e6:.0f} MB (> 126 MB L2) between reuses"},
        "secondary": {
            "decode_m8_gbs": None if gbs8 is None else round(gbs8, 2),
            "prefill_m512_tflops": round(tflops_p, 2),
            "prefill_m512_frac_of_bf16_peak": round(tflops_p / tc_peak, 4),
            "prefill_m512_us_per_op": round(msp * 1e3 / (max(1, args.steps // 4) * Rp), 3),
            "configs_1_2_device_us_per_op": {o["case"]: round(o["graph_us_per_call"], 3) for o in ops_lines},
            "conv_through_gemm_cores": conv_line,
            "config5_decoder": dec_line,
            "config4_bert": bert_line,
        },
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                     else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_launch": launch_bytes(1)},
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "h2d_bytes_per_step": e2e_layers * K_DIM * 4,
                "d2h_bytes_per_step": e2e_layers * N_DIM * 4,
                "what": f"b2m_matmul_nbits_host per layer ({e2e_layers} layers per step): pinned A -> device, "
                        "kernel, Y -> pinned host, synchronise"},
        "gpu_launches": args.steps * R * P,
        "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if cpu_all is not None:
        line["secondary"]["cpu_baselines_per_config"] = cpu_all
    if rank == 0:
        print(json.dumps(line), flush=True)
    for w in packed:
        w.free()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
