#!/usr/bin/env python3
"""Benchmark driver: one JSON line on rank 0.

Default workload (the metric's T2S decode): batch-1
greedy decode of the 24-layer d=512 T2S transformer, KV prefix of 256 slots,
64-token prompt, 500 tokens per utterance.  A "step" is one utterance: prompt
prefill + 500 greedy steps.  Multi-GPU runs are replicas (one utterance per
GPU per step, no collective on the data path): value = tokens of all ranks /
max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gsvk|reference]
                  [--workload t2s_decode_b1|gemm_ffn_up]

--impl reference times the reference's CPU arithmetic for the same workload on
the host cores (the oracle restatement; the reference itself targets Apple
NEON/Accelerate and does not build on x86).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

T2S_STEPS = 500
# DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) of one decode
# launch divided by its algorithmic bytes, measured on a 20-step launch of the
# default decode kernel (t2s_flow_kernel: 3.1665 GB against 3.1980 GB);
# traffic grows in proportion to the decode passes.
T2S_TRAFFIC_RATIO = 0.990
T2S_PREFIX = 256
T2S_PROMPT = 64
L2_BYTES = 126 * 1024 * 1024


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # sampling is running once the first row is out (bounded: 3 s)
        deadline = time.time() + 3.0
        while time.time() < deadline and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((int(parts[0]), float(parts[1]), float(parts[2]), parts[4:]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        max_mhz = max(r[2] for r in rows)
        loaded = [r for r in rows if r[1] >= 0.5 * r[2]] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3][1:5])
                          if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[1] for r in loaded), "sm_max_mhz": max_mhz,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------- distributed
# One process per GPU; the package's replicas module holds the host logic
# (NCCL only for barriers, the max-over-ranks time and result gathering).
def _replicas():
    return __import__("__graft_entry__").package().replicas


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch

        torch.cuda.set_device(local)
        _replicas().init("nccl", rank, world, device=torch.device("cuda", local))
    return rank, local, world


def barrier(world):
    _replicas().barrier(world)


def max_over_ranks(v, world):
    return _replicas().max_over_ranks(v, world, device="cuda" if world > 1 else None)


def dist_close(world):
    _replicas().close(world)


# --------------------------------------------- workload identity (both arms)
# metric, unit and config of every workload: the GPU arm and the reference
# arm print the same ones.
def workload_meta(args, world):
    import numpy as np

    W = __import__("__graft_entry__").package().workloads
    wl = args.workload
    if wl == "t2s_decode_b1":
        return dict(metric="T2S decode tokens/s (batch 1 per GPU, 500 greedy tokens per utterance)",
                    unit="tokens/s", dtype="f16 weights/KV, f32 accumulate",
                    data="synthetic (seeded N(0,0.02) weights, N(0,1) KV prefix, uniform prompt ids)",
                    config={"workload": "t2s_decode_b1 (BASELINE configs[1])",
                            "model": "T2S 24L d512 16h ffn2048 vocab1025 post-LN",
                            "global_batch": world, "seq_len": T2S_STEPS, "kv_prefix": T2S_PREFIX,
                            "prompt": T2S_PROMPT, "parallelism": f"replicas x{world}",
                            "l2": "inputs larger than L2: 152 MB of weights streamed per token"})
    if wl == "gemm_ffn_up":
        return dict(metric="GEMM TFLOP/s (Y = ReLU(X W^T + b), 128x2048x512, fp16 out)",
                    unit="TFLOP/s", dtype="f16 in, f32 accumulate, f16 out", data="synthetic",
                    config={"workload": "gemm_ffn_up (BASELINE configs[0])", "shape": [128, 2048, 512],
                            "epilogue": "bias + ReLU, fp16 out", "global_batch": world,
                            "parallelism": f"replicas x{world}",
                            "l2": "128 X/W/Y copies per launch (weights 268 MB > L2)"})
    if wl == "gemm":
        M, N, K = (int(v) for v in args.gemm_shape.split(","))
        return dict(metric=f"GEMM TFLOP/s ({M}x{N}x{K}, fp16 out)", unit="TFLOP/s",
                    dtype="f16 in, f32 accumulate, f16 out", data="synthetic N(0,1) x N(0,0.02)",
                    config={"workload": "gemm", "shape": [M, N, K], "global_batch": world,
                            "parallelism": f"replicas x{world}",
                            "l2": "rotated operand copies > L2"})
    if wl == "sovits_decoder":
        cfg = W.DECODER
        return dict(metric="SoVITS decoder TFLOP/s (192x500 latent -> 320,000 samples per utterance)",
                    unit="TFLOP/s", dtype="f16 activations/weights, f32 accumulate and residual",
                    data="synthetic (N(0,0.01) weights, N(0,1) latent)",
                    config={"workload": "sovits_decoder (BASELINE configs[4])", "frames": 500,
                            "samples": 500 * int(np.prod(cfg["up_rate"])), "global_batch": world,
                            "parallelism": f"replicas x{world}",
                            "l2": "activations 20-40 MB per layer at the late stages, > L2 per step"})
    if wl == "encoder":
        e = W.ENCODERS[args.encoder]
        return dict(metric=f"{args.encoder} encoder prefill GEMM TFLOP/s (batch {e['batch']} x {e['seq']})",
                    unit="TFLOP/s", dtype="f16 operands, f32 accumulate",
                    data="synthetic (N(0,0.02) weights, N(0,1) activations)",
                    config={"workload": f"encoder_{args.encoder} (BASELINE configs[3])",
                            "layers": e["layers"], "hidden": e["hidden"], "ffn": e["ffn"],
                            "global_batch": e["batch"] * world, "seq_len": e["seq"],
                            "parallelism": f"replicas x{world}",
                            "flops_counted": "the stack's GEMM FLOPs; time is the whole forward",
                            "l2": "weights 0.2-0.6 GB and activations > L2 per step"})
    if wl == "t2s_decode_b64":
        B = args.batch
        lens = W.t2s_batched_lengths(B, seed=1)
        return dict(metric=f"batched T2S decode tokens/s ({B} utterances per GPU)", unit="tokens/s",
                    dtype="f16 operands, f32 accumulate",
                    data="synthetic (N(0,0.02) weights, N(0,1) KV, lengths U{64..1024} seed 1)",
                    config={"workload": "t2s_decode_b64 (BASELINE configs[2])", "batch": B,
                            "decode_steps_per_step": 32, "mean_kv_len": float(lens.mean()),
                            "global_batch": B * world, "parallelism": f"replicas x{world}",
                            "l2": "1.9 GB of weights + KV streamed per decode step"})
    if wl in ENGINE_WORKLOADS:
        d = ENGINE_WORKLOADS[wl]
        return dict(metric=d["metric"], unit="TFLOP/s", dtype=d["dtype"], data=d["data"],
                    config={"workload": wl, **d["shape"], "global_batch": world,
                            "parallelism": f"replicas x{world}",
                            "l2": "a 256 MB buffer written between timed forwards (L2 flushed)",
                            "flops_counted": "conv / GEMM / attention products; time is the "
                                             "whole forward"})
    if wl == "gemv_t2s":
        return dict(metric="T2S GEMV GB/s (one token's 97 GEMVs: 24 x {1536x512, 512x512, "
                           "2048x512, 512x2048} + 1025x512)",
                    unit="GB/s", dtype="f16 weights, f32 x and accumulate",
                    data="synthetic (seeded N(0,0.02) weights, N(0,1) x)",
                    config={"workload": "gemv_t2s (the T2S decode GEMV shapes)",
                            "launch": "CUDA graph of one token's 97 gemv_f16w_f32acc launches",
                            "global_batch": world, "parallelism": f"replicas x{world}",
                            "l2": f"{GEMV_SETS} rotated copies of the 152 MB weight set (> L2)"})
    raise ValueError(wl)


# ----------------------------------------------------- CPU baseline (oracle)
# The reference is Apple-only (NEON, Accelerate, AArch64 AMX) and does not
# build here, so its CPU arithmetic is timed through the oracle restatement
# (kind "port"), threaded over the host cores.  Every workload has a bounded
# sample of its own work; a sample is timed whole and reported as the
# workload's unit.

def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sampler(args, threads):
    """(fn, units_per_call, description): fn() runs one bounded sample of the
    workload on the oracle; units_per_call is in the workload's unit
    numerator (tokens, or FLOPs for TFLOP/s)."""
    import numpy as np
    import oracle

    W = __import__("__graft_entry__").package().workloads
    oracle.build()
    oracle.set_threads(threads)
    wl = args.workload
    if wl == "t2s_decode_b1":
        m = W.t2s_model(seed=0)
        L, D = m["n_layers"], m["d_model"]
        top = T2S_PREFIX + T2S_PROMPT + T2S_STEPS
        kc, vc = W.t2s_kv_prefix(m, top + 1, top, seed=5)
        ctxs = [int(c) for c in np.linspace(T2S_PREFIX + T2S_PROMPT + 1, top, 10)]
        hist = np.arange(64, dtype=np.int32)

        def fn():
            tok = 7
            for c in ctxs:  # one decode token at each of 10 context lengths over 321..820
                pe = oracle.t2s_pe_row(D, c - T2S_PREFIX)
                x = (pe + m["audio_emb"][tok].view(np.float16).astype(np.float32)).astype(np.float32)
                for layer in range(L):
                    oracle.t2s_decode_layer(m, layer, x, c, kc[layer], vc[layer])
                lg = oracle.gemv_f16w_f32acc(m["wpred"], x)
                tok, _ = oracle.t2s_greedy_sample(lg, hist, True)
        return fn, len(ctxs), ("oracle T2S decode: one token (24 layers, logits, sampling) at each of "
                               f"10 context lengths evenly spaced over {ctxs[0]}..{ctxs[-1]}; the "
                               "64-token prompt prefill is not in the sample")
    if wl in ("gemm_ffn_up", "gemm"):
        if wl == "gemm_ffn_up":
            x, w, b = W.gemm_ffn_up(seed=0)
            M, N, K = 128, 2048, 512
            act = oracle.ACT_RELU
        else:
            M, N, K = (int(v) for v in args.gemm_shape.split(","))
            M = min(M, 256)  # row band sample of a large shape
            rng = np.random.default_rng(0)
            x = W._f16(rng.standard_normal((M, K), dtype=np.float32))
            w = W._f16(rng.standard_normal((N, K), dtype=np.float32) * 0.02)
            b, act = None, oracle.ACT_NONE
        xf = x.view(np.float16).astype(np.float32)
        reps = 4

        def fn():
            for _ in range(reps):
                oracle.linear_f16(xf, w, b, act)
        return fn, 2 * M * N * K * reps, (f"oracle gemm_f16x_fmlal order, {reps} x "
                                         f"{M}x{N}x{K} with the fused epilogue")
    if wl == "encoder":
        e = W.ENCODERS[args.encoder]
        ub, T = 4, e["seq"]
        m = W.encoder_model(args.encoder, layers=1, seed=0)
        x = W.encoder_input(args.encoder, batch=ub, seq=T, seed=0)
        C, F = e["hidden"], e["ffn"]

        def fn():
            oracle.encoder_layer(m, 0, x.copy(), ub, T, None)
        return fn, 2 * ub * T * (4 * C * C + 2 * C * F), (
            f"oracle {args.encoder} layer (full post-LN layer) on {ub} of the {e['batch']} "
            f"utterances x {T}; FLOPs counted as the layer's GEMMs")
    if wl == "sovits_decoder":
        cfg = W.DECODER
        ws, bs = W.decoder_weights(cfg, seed=0)
        T = 40
        z = W.decoder_latent(T, cfg, seed=0)
        dc = oracle.decoder_cfg(**cfg)

        def fn():
            oracle.decoder_forward(dc, ws, bs, z, round_in=True)
        return fn, 2 * W.decoder_macs(cfg, T), f"oracle generator on a {T}-frame latent (of 500)"
    if wl == "t2s_decode_b64":
        m = W.t2s_model(seed=1)
        L, D = m["n_layers"], m["d_model"]
        lens = W.t2s_batched_lengths(args.batch, seed=1)[:8]
        caches = [W.t2s_kv_prefix(m, int(n) + 1, int(n), seed=600 + i) for i, n in enumerate(lens)]
        hist = np.arange(8, dtype=np.int32)

        def fn():
            for (kc, vc), n in zip(caches, lens):
                x = m["audio_emb"][3].view(np.float16).astype(np.float32)
                for layer in range(L):
                    oracle.t2s_decode_layer(m, layer, x, int(n), kc[layer], vc[layer])
                lg = oracle.gemv_f16w_f32acc(m["wpred"], x)
                oracle.t2s_greedy_sample(lg, hist, True)
        return fn, len(lens), (f"oracle T2S decode: one token for each of the first {len(lens)} "
                               f"utterances (KV lengths {', '.join(str(int(v)) for v in lens)})")
    if wl in ENGINE_WORKLOADS:
        fn, flops, desc = engine_cpu_sample(wl, W, oracle)
        return fn, flops, desc
    if wl == "gemv_t2s":
        m = W.t2s_model(seed=0)
        x = np.random.default_rng(0).standard_normal(2048).astype(np.float32)
        mats = [m[k][i] for i in range(m["n_layers"]) for k in ("wqkv", "wout", "w1", "w2")]
        mats.append(m["wpred"])

        def fn():
            for w in mats:
                oracle.gemv_f16w_f32acc(w, x[:w.shape[1]])
        return fn, sum(w.nbytes for w in mats) / 1e9, (
            "oracle gemv_f16w_f32acc over one token's 97 weight matrices (152 MB)")
    raise ValueError(wl)


def cpu_measure(args, warmup=2, samples=7, threads=None):
    """Median of `samples` timed samples after `warmup`; returns the
    cpu_baseline dict (value in the workload's unit)."""
    threads = threads or (os.cpu_count() or 1)
    fn, units, desc = cpu_sampler(args, threads)
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(samples):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return cpu_result(args, units, desc, times, threads)


def cpu_result(args, units, desc, times, threads):
    meta = workload_meta(args, 1)
    med = statistics.median(times)
    scale = 1e-12 if meta["unit"] == "TFLOP/s" else 1.0
    cv = statistics.pstdev(times) / statistics.mean(times) * 100 if len(times) > 1 else 0.0
    return {"value": units / med * scale, "unit": meta["unit"], "cores": threads, "kind": "port",
            "sample": f"{desc}; median of {len(times)} samples ({med * 1e3:.1f} ms each, "
                      f"CV {cv:.1f} %)",
            "median_ms": med * 1e3, "cv_pct": cv, "n_samples": len(times),
            "nproc": os.cpu_count(), "cpu_model": cpu_model()}


# ------------------------------------------------------------ T2S workload
def t2s_algorithmic_bytes(model, steps):
    """HBM bytes the decode kernel must move: per decode pass all weights
    (24 x 6,291,456 + logits 1,049,600 B) + K/V reads over len slots
    (49,152 B per slot) + K/V writes (49,152 B)."""
    L, D, F, V = model["n_layers"], model["d_model"], model["ffn"], model["vocab"]
    w = L * (3 * D * D + D * D + 2 * F * D) * 2 + V * D * 2
    kv_slot = L * 2 * D * 2
    total = 0
    for i in range(steps - 1):  # the last step only samples
        length = T2S_PREFIX + T2S_PROMPT + i + 1
        total += w + kv_slot * length + kv_slot
    return total


def run_t2s(args, rank, local, world):
    import numpy as np
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    m, k0, v0, _ = g.workloads.t2s_decode_b1()
    prompt = g.workloads.t2s_prompt(T2S_PROMPT, m["vocab"], seed=rank)  # one utterance per rank
    cap = T2S_PREFIX + T2S_PROMPT + T2S_STEPS
    eng = g.T2S(m, cap)
    if args.decode_kernel:
        eng.set_decode_kernel(args.decode_kernel)
    k_pin = torch.from_numpy(k0[:, :T2S_PREFIX].copy()).pin_memory()
    v_pin = torch.from_numpy(v0[:, :T2S_PREFIX].copy()).pin_memory()
    eng.load_kv(k_pin.numpy(), v_pin.numpy(), T2S_PREFIX)
    prompt_dev = torch.from_numpy(prompt).to(dev)
    toks = torch.zeros(T2S_STEPS, dtype=torch.int32, device=dev)
    nout = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)

    def step():
        eng.prompt(T2S_PREFIX, prompt_dev)
        eng.decode(T2S_PREFIX, prompt_dev, T2S_STEPS, toks, nout, stop_on_eos=False)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    assert g.device_status() == 0

    # ---- device-resident timing (value) + per-launch decode kernel events
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    barrier(world)
    torch.cuda.synchronize(dev)
    clocks.start()
    start.record(stream)
    for i in range(args.steps):
        eng.prompt(T2S_PREFIX, prompt_dev)
        ev[i][0].record(stream)
        eng.decode(T2S_PREFIX, prompt_dev, T2S_STEPS, toks, nout, stop_on_eos=False)
        ev[i][1].record(stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    barrier(world)
    t_total = start.elapsed_time(end) * 1e-3
    t_dec = statistics.mean(a.elapsed_time(b) for a, b in ev) * 1e-3
    assert int(nout.item()) == T2S_STEPS and g.device_status() == 0
    t_max = max_over_ranks(t_total, world)
    t_dec_max = max_over_ranks(t_dec, world)

    # ---- end to end through the C-ABI with host buffers (e2e)
    h2d = k_pin.numel() * 2 * 2 + prompt.nbytes
    d2h = T2S_STEPS * 4 + 4
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        eng.load_kv(k_pin.numpy(), v_pin.numpy(), T2S_PREFIX)
        out, _ = eng.generate(T2S_PREFIX, prompt, T2S_STEPS, stop_on_eos=False)
        assert len(out) == T2S_STEPS
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
    launches = eng.launches_per_generate() * args.steps
    kernel_name = {1: "t2s_decode_kernel", 2: "t2s_cluster_kernel",
                   3: "t2s_flow_kernel"}[eng.decode_kernel()]
    eng.close()

    tokens = T2S_STEPS * args.steps * world
    hbm, _, peak_kind = measured_peaks()
    alg = t2s_algorithmic_bytes(m, T2S_STEPS)
    achieved = alg / t_dec_max / 1e9
    line = {
        "metric": "T2S decode tokens/s (batch 1 per GPU, 500 greedy tokens per utterance)",
        "value": tokens / t_max,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_max / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 weights/KV, f32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV prefix, uniform prompt ids)",
        "config": {"workload": "t2s_decode_b1 (BASELINE configs[1])",
                   "model": "T2S 24L d512 16h ffn2048 vocab1025 post-LN",
                   "global_batch": world, "seq_len": T2S_STEPS, "kv_prefix": T2S_PREFIX,
                   "prompt": T2S_PROMPT, "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: 152 MB of weights streamed per token"},
        "e2e": {"value": tokens / t_e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": kernel_name, "achieved": achieved,
                     "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": peak_kind, "traffic": T2S_TRAFFIC_RATIO * alg,
                     "traffic_note": "ncu DRAM bytes of a 20-step launch of the same kernel, "
                                     "scaled per pass (profiles/t2s_flow_kernel_config2.md)",
                     "algorithmic_bytes_per_launch": alg,
                     "launch_ms": t_dec_max * 1e3},
    }
    if clk:
        line["clocks"] = clk
    return line


# ------------------------------------------------------------ GEMM config 1
def run_gemm1(args, rank, local, world):
    import numpy as np
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    x, w, b = g.workloads.gemm_ffn_up(seed=rank)
    # 128 independent instances per launch (gsvk_gemm_f16_batched: one
    # persistent tensor-core launch over every problem's tiles), each on its
    # own X / W / Y; the 128 weight copies (268 MB) exceed L2.
    batch, iters, sets = 128, 1024, 1
    x16 = torch.from_numpy(x.view(np.float16)).to(dev)
    w16 = torch.from_numpy(w.view(np.float16)).to(dev)
    xs = [x16.unsqueeze(0).repeat(batch, 1, 1).contiguous() for _ in range(sets)]
    ws = [w16.unsqueeze(0).repeat(batch, 1, 1).contiguous() for _ in range(sets)]
    bd = torch.from_numpy(b).to(dev)
    ys = [torch.empty(batch, 128, 2048, dtype=torch.float16, device=dev) for _ in range(sets)]
    for i in range(sets):
        g.gemm_batched(xs[i], ws[i], bias=bd, act=g.ACT_RELU, c_f16=ys[i])
    torch.cuda.synchronize(dev)
    # Steady state: iters / batch back-to-back launches captured in one CUDA
    # graph (268 MB of weights between reuses).
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for j in range(iters // batch):
            g.gemm_batched(xs[j % sets], ws[j % sets], bias=bd, act=g.ACT_RELU, c_f16=ys[j % sets])
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    start.record(stream)
    for s in range(args.steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(start.elapsed_time(end) * 1e-3, world)
    # e2e: every launch's activations from pinned host memory and its outputs
    # back to the host (weights stay resident)
    x_pin = xs[0].cpu().pin_memory()
    y_pin = torch.empty(ys[0].shape, dtype=torch.float16).pin_memory()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        for j in range(iters // batch):
            xs[0].copy_(x_pin, non_blocking=True)
            g.gemm_batched(xs[0], ws[0], bias=bd, act=g.ACT_RELU, c_f16=ys[0])
            y_pin.copy_(ys[0], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
    flops = 2 * 128 * 2048 * 512 * iters * args.steps * world
    hbm, tf, kind = measured_peaks()
    alg_bytes = 2760704  # X 131,072 + W 2,097,152 + b 8,192 + Y 524,288 per GEMM
    achieved_gbs = alg_bytes * iters * args.steps / t / 1e9
    line = {"metric": "GEMM TFLOP/s (Y = ReLU(X W^T + b), 128x2048x512, fp16 out)",
            "value": flops / t / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 in, f32 accumulate, f16 out",
            "data": "synthetic", "config": {"workload": "gemm_ffn_up (BASELINE configs[0])",
                                            "iters_per_step": iters,
                                            "launch": f"CUDA graph of {iters // batch} strided-batched launches of {batch} independent GEMMs (gsvk_gemm_f16_batched)",
                                            "l2": f"{batch} X/W/Y copies per launch (weights 268 MB > L2)"},
            "e2e": {"value": flops / t_e2e / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x_pin.numel() * 2 * (iters // batch),
                    "d2h_bytes_per_step": y_pin.numel() * 2 * (iters // batch),
                    "note": "bound by the host link: 134 MB in and 537 MB out per 1024 GEMMs"},
            "gpu_launches": iters // batch * args.steps,
            "roofline": {"bound": "hbm", "kernel": "gemm_tc_kernel (strided batch)",
                         "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s",
                         "frac": achieved_gbs / hbm, "peak_source": kind, "traffic": None,
                         "algorithmic_bytes_per_gemm": alg_bytes,
                         "tensor_frac": flops / world / t / 1e12 / tf,
                         "note": "AI 97 flop/B is below the ridge: HBM-bound"}}
    if clk:
        line["clocks"] = clk
    return line


# ---------------------------------- SoVITS latent path, SV, HuBERT front-end
ENGINE_WORKLOADS = {
    "hubert_front": dict(
        metric="HuBERT front-end TFLOP/s (10 s of 16 kHz audio per forward)",
        dtype="f16 operands, f32 accumulate", shape={"samples": 160000},
        data="synthetic (N(0,0.1) waveform, N(0,1/fan_in) conv weights)"),
    "sovits_latent": dict(
        metric="SoVITS latent path TFLOP/s (250 codes = 500 frames, 100 phones per forward)",
        dtype="f16 conv operands, f32 accumulate and attention", shape={"codes": 250, "phones": 100},
        data="synthetic (uniform codes / phones, N(0,1/fan_in) conv weights, N(0,1) noise)"),
    "sv": dict(
        metric="SV encoder TFLOP/s (500 fbank frames per forward)",
        dtype="f16 conv operands, f32 accumulate, fp64 BatchNorm", shape={"frames": 500},
        data="synthetic (N(0,1) fbank, He-initialised convs)"),
}


def hubert_front_flops(cfg, n):
    t, ci, f = n, 1, 0
    for co, k, s in zip(cfg["conv_dim"], cfg["conv_kernel"], cfg["conv_stride"]):
        t = (t - k) // s + 1
        f += 2 * t * co * ci * k
        ci = co
    H = cfg["hidden"]
    return f + 2 * t * H * ci + 2 * t * H * (H // cfg["pos_groups"]) * cfg["pos_k"]


def sovits_latent_flops(c, n_codes, n_phones):
    Tq, Tt, C, F, MH = 2 * n_codes, n_phones, c["hidden"], c["filter"], c["mrte_hidden"]
    K = c["kernel"]

    def enc(T, L):
        return L * (2 * T * 3 * C * C + 4 * T * T * C + 2 * T * C * C + 4 * T * F * C * K)

    f = 2 * Tq * C * c["ssl_dim"] + enc(Tq, c["layers_ssl"]) + enc(Tt, c["layers_text"])
    f += enc(Tq, c["layers_2"])
    f += 2 * Tq * MH * C + 2 * Tt * MH * C + 2 * Tq * MH * MH + 4 * Tt * MH * MH
    f += 4 * Tq * Tt * MH + 2 * Tq * MH * MH + 2 * Tq * C * MH + 4 * Tq * C * C
    nl = c["wn_layers"]
    per_flow = 2 * Tq * C * (C // 2) + 4 * C * nl * c["gin"] + 2 * Tq * (C // 2) * C
    per_flow += sum(2 * Tq * 2 * C * C * c["wn_kernel"] + 2 * Tq * (2 * C if l + 1 < nl else C) * C
                    for l in range(nl))
    return f + c["flows"] * per_flow


def sv_flops(frames, n_mels=80, m_ch=64, base_width=24, scale=4, expansion=4, stages=None):
    stages = stages or __import__("__graft_entry__").package().workloads.SV_STAGES
    h, w = n_mels, frames
    f = 2 * h * w * m_ch * 9
    c = m_ch
    for l, (blocks, stride, aff) in enumerate(stages, 1):
        planes = m_ch * 2 ** (l - 1)
        width, exp = planes * base_width // 64, planes * expansion
        for i in range(blocks):
            st = stride if i == 0 else 1
            h, w = (h - 1) // st + 1, (w - 1) // st + 1
            S, co1 = h * w, width * scale
            f += 2 * S * co1 * c + scale * 2 * S * width * width * 9 + 2 * S * exp * co1
            if aff:
                inter = width // 4
                f += (scale - 1) * (2 * S * inter * 2 * width + 2 * S * width * inter)
            if i == 0 and (st != 1 or c != exp):
                f += 2 * S * exp * c
            c = exp
        if l == 3:
            c3 = c
    S4 = h * w
    return f + 2 * S4 * c * c3 * 9 + 2 * S4 * (c // 4) * 2 * c + 2 * S4 * c * (c // 4)


def engine_setup(wl, g, dev):
    """(forward(), e2e_step(), flops, h2d_bytes, d2h_bytes) for one engine
    workload; inputs resident on `dev`, pinned host copies for e2e."""
    import numpy as np
    import torch

    W = g.workloads
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()  # noqa: E731
    if wl == "hubert_front":
        n = ENGINE_WORKLOADS[wl]["shape"]["samples"]
        m = W.hubert_front_model(seed=0)
        fe = g.HubertFront(m, max_samples=n)
        wav_h = pin(W.hubert_waveform(n, seed=0))
        wav = wav_h.to(dev)
        x = torch.empty(fe.frames(n), m["hidden"], device=dev)
        x_h = torch.empty(x.shape).pin_memory()

        def e2e():
            wav.copy_(wav_h, non_blocking=True)
            fe.forward(wav, x)
            x_h.copy_(x, non_blocking=True)
        return (lambda: fe.forward(wav, x)), e2e, hubert_front_flops(m, n), n * 4, x.numel() * 4, fe
    if wl == "sovits_latent":
        sh = ENGINE_WORKLOADS[wl]["shape"]
        m = W.sovits_latent_model(seed=0)
        eng = g.SovitsLatent(m, sh["codes"], sh["phones"])
        codes, phones, ge, ge_text, nz = W.sovits_latent_inputs(sh["codes"], sh["phones"], seed=0)
        hs = [pin(a) for a in (ge, ge_text, nz)]
        ds = [h.to(dev) for h in hs]
        z = torch.empty(m["hidden"], 2 * sh["codes"], device=dev)
        z_h = torch.empty(z.shape).pin_memory()

        def e2e():
            for d_, h_ in zip(ds, hs):
                d_.copy_(h_, non_blocking=True)
            eng.forward(codes, phones, *ds, z=z)
            z_h.copy_(z, non_blocking=True)
        h2d = sum(h.numel() * 4 for h in hs) + codes.nbytes + phones.nbytes
        return ((lambda: eng.forward(codes, phones, *ds, z=z)), e2e,
                sovits_latent_flops(m, sh["codes"], sh["phones"]), h2d, z.numel() * 4, eng)
    if wl == "sv":
        T = ENGINE_WORKLOADS[wl]["shape"]["frames"]
        m = W.sv_model(seed=0)
        enc = g.SvEncoder(m, max_frames=T)
        fb_h = pin(W.sv_fbank(T, seed=0))
        fb = fb_h.to(dev)
        emb = torch.empty(enc.embedding_size(), device=dev)
        emb_h = torch.empty(emb.shape).pin_memory()

        def e2e():
            fb.copy_(fb_h, non_blocking=True)
            enc.forward(fb, emb)
            emb_h.copy_(emb, non_blocking=True)
        return (lambda: enc.forward(fb, emb)), e2e, sv_flops(T), fb.numel() * 4, emb.numel() * 4, enc
    raise ValueError(wl)


def engine_cpu_sample(wl, W, oracle):
    """A bounded oracle sample of an engine workload: (fn, flops, description)."""
    if wl == "hubert_front":
        m = W.hubert_front_model(seed=0)
        wav = W.hubert_waveform(16000, seed=0)
        return (lambda: oracle.hubert_front(m, wav)), hubert_front_flops(m, 16000), \
            "oracle HuBERT front-end on 1 s of audio (of 10 s)"
    if wl == "sovits_latent":
        m = W.sovits_latent_model(seed=0)
        inp = W.sovits_latent_inputs(50, 40, seed=0)
        return (lambda: oracle.sovits_latent(m, *inp)), sovits_latent_flops(m, 50, 40), \
            "oracle SoVITS latent path on 50 codes / 40 phones (of 250 / 100)"
    if wl == "sv":
        m = W.sv_model(seed=0)
        fb = W.sv_fbank(16, seed=0)
        return (lambda: oracle.sv_forward(m, fb)), sv_flops(16), \
            "oracle SV encoder on 16 fbank frames (of 500)"
    raise ValueError(wl)


def count_kernels(fn):
    """Kernels one call of fn launches, from the CUDA profiler's activity
    records (None when the profiler is unavailable)."""
    import torch

    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and
                   not e.name.lower().startswith(("memcpy", "memset")))
    except Exception:
        return None


def run_engine(args, rank, local, world):
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    fwd, e2e, flops, h2d, d2h, keep = engine_setup(args.workload, g, dev)
    flush = torch.empty(64 << 20, device=dev)  # 256 MB > L2
    for _ in range(args.warmup):
        fwd()
    torch.cuda.synchronize(dev)
    launches = None if args.no_launch_count else count_kernels(fwd)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        fwd()
        b.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) * 1e-3 / args.steps, world)
    barrier(world)
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        e2e()
        b.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) * 1e-3 / args.steps, world)
    hbm, tf, kind = measured_peaks()
    value = flops * world / t / 1e12
    line = {"metric": ENGINE_WORKLOADS[args.workload]["metric"], "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "e2e": {"value": flops * world / t_e2e / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": t_e2e * 1e3},
            "gpu_launches": None if launches is None else launches * args.steps,
            "roofline": {"bound": "tensor", "kernel": "whole forward (conv GEMMs dominate)",
                         "achieved": value / world, "peak": tf, "unit": "TFLOP/s",
                         "frac": value / world / tf, "peak_source": kind, "traffic": None,
                         "flops_per_forward": flops,
                         "note": "small per-utterance shapes: launch- and latency-bound"}}
    if clk:
        line["clocks"] = clk
    del keep
    return line


# ------------------------------------------------ T2S GEMV shapes (a1, a2)
GEMV_SETS = 4
GEMV_SHAPES = ((1536, 512), (512, 512), (2048, 512), (512, 2048), (1025, 512))


def run_gemv_t2s(args, rank, local, world):
    """One token's GEMVs as standalone gemv_f16w_f32acc launches (the a1
    kernel at the five T2S shapes), GEMV_SETS rotated weight sets so every
    launch streams its weights from HBM; then, per shape, the same kernel on
    its own over >= 256 MB of rotated copies, and the M=64 product through
    the tensor-core skinny GEMM against 64 fp16-x GEMV launches."""
    import numpy as np
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    m = g.workloads.t2s_model(seed=rank)
    L = m["n_layers"]
    names = ("wqkv", "wout", "w1", "w2")
    base = [torch.from_numpy(m[k][i].view(np.float16)).to(dev) for i in range(L) for k in names]
    base.append(torch.from_numpy(m["wpred"].view(np.float16)).to(dev))
    sets = [[w.clone() for w in base] for _ in range(GEMV_SETS)]
    x = torch.randn(2048, device=dev)
    ys = [torch.empty(w.shape[0], device=dev) for w in base]
    tok_bytes = sum(w.numel() * 2 + w.shape[1] * 4 + w.shape[0] * 4 for w in base)

    def token(ws):
        for w, y in zip(ws, ys):
            g.gemv_f16w_f32acc(w, x[:w.shape[1]], y)

    token(sets[0])
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for ws in sets:
            token(ws)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    start.record(stream)
    for _ in range(args.steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(start.elapsed_time(end) * 1e-3, world)
    launches = len(base) * GEMV_SETS * args.steps
    value = tok_bytes * GEMV_SETS * args.steps * world / t / 1e9
    # e2e: x from pinned host memory and every y back to it, per token
    x_pin = x.cpu().pin_memory()
    y_pin = torch.empty(sum(y.numel() for y in ys)).pin_memory()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for ws in sets:
            x.copy_(x_pin, non_blocking=True)
            token(ws)
            o = 0
            for y in ys:
                y_pin[o:o + y.numel()].copy_(y, non_blocking=True)
                o += y.numel()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)
    del graph, sets
    torch.cuda.empty_cache()
    hbm, tf, kind = measured_peaks()
    shapes = {}
    for N, K in GEMV_SHAPES:
        wb = N * K * 2
        R = max(4, -(-(256 << 20) // wb))
        ws = torch.randn(R, N, K, device=dev).mul_(0.02).half()
        xv, xh = torch.randn(K, device=dev), torch.randn(64, K, device=dev).half()
        y, y64 = torch.empty(N, device=dev), torch.empty(64, N, device=dev)
        reps = 256
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for j in range(reps):
                g.gemv_f16w_f32acc(ws[j % R], xv, y)
        gr.replay()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(4):
            gr.replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
        us1 = a.elapsed_time(b) * 1e3 / (4 * reps)
        gb1 = (wb + K * 4 + N * 4) / us1 / 1e3
        # M = 64: one skinny tensor-core GEMM vs 64 fp16-x GEMV launches
        tc = torch.cuda.CUDAGraph()
        with torch.cuda.graph(tc):
            for j in range(64):
                g.gemm_ex(xh, ws[j % R], c=y64)
        gv = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gv):
            for j in range(8):
                for r in range(64):
                    g.gemv_f16x_fmlal(ws[j % R], xh[r], y64[r])
        res = []
        for gg, n in ((tc, 64), (gv, 8)):
            gg.replay()
            torch.cuda.synchronize(dev)
            a.record(stream)
            for _ in range(4):
                gg.replay()
            b.record(stream)
            torch.cuda.synchronize(dev)
            res.append(a.elapsed_time(b) * 1e3 / (4 * n))
        shapes[f"{N}x{K}"] = {"copies": R, "gemv_us": round(us1, 3), "gemv_gbs": round(gb1, 1),
                              "gemv_frac": round(gb1 / hbm, 4),
                              "m64_tensor_us": round(res[0], 3), "m64_gemv_x64_us": round(res[1], 3)}
        del ws, gr, tc, gv
        torch.cuda.empty_cache()
    line = {"metric": workload_meta(args, world)["metric"], "value": value, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "e2e": {"value": tok_bytes * GEMV_SETS * args.steps * world / t_e2e / 1e9,
                    "unit": "GB/s", "h2d_bytes_per_step": x_pin.numel() * 4 * GEMV_SETS,
                    "d2h_bytes_per_step": y_pin.numel() * 4 * GEMV_SETS},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": "gemv_vec_kernel", "achieved": value / world,
                         "peak": hbm, "unit": "GB/s", "frac": value / world / hbm,
                         "peak_source": kind, "traffic": None,
                         "algorithmic_bytes_per_token": tok_bytes},
            "shapes": shapes}
    if clk:
        line["clocks"] = clk
    return line


# ------------------------------------------- one GEMM shape, back to back
def run_gemm_shape(args, rank, local, world):
    """C = A B^T for --gemm-shape M,N,K (fp16 in, fp32 accumulate, fp16 out),
    captured as 100 launches in a CUDA graph per step, rotating enough
    operand copies that the working set exceeds L2."""
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    M, N, K = (int(v) for v in args.gemm_shape.split(","))
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    per = (M * K + N * K + M * N) * 2
    copies = max(1, min(8, -(-256 * 2 ** 20 // per)))
    a = [torch.randn(M, K, device=dev, generator=gen).half() for _ in range(copies)]
    w = [(torch.randn(N, K, device=dev, generator=gen) * 0.02).half() for _ in range(copies)]
    c = [torch.empty(M, N, device=dev, dtype=torch.float16) for _ in range(copies)]
    iters = 100
    for i in range(copies):
        g.gemm_ex(a[i], w[i], c_f16=c[i])
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(iters):
            g.gemm_ex(a[i % copies], w[i % copies], c_f16=c[i % copies])
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    start.record(stream)
    for _ in range(args.steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(start.elapsed_time(end) * 1e-3, world)
    flops = 2.0 * M * N * K * iters * args.steps
    _, tf, kind = measured_peaks()
    achieved = flops / t / 1e12
    line = {"metric": f"GEMM TFLOP/s ({M}x{N}x{K}, fp16 out)", "value": achieved * world,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 in, f32 accumulate, f16 out", "data": "synthetic N(0,1) x N(0,0.02)",
            "config": {"workload": "gemm", "shape": [M, N, K], "iters_per_step": iters,
                       "launch": "CUDA graph", "l2": f"{copies} rotated operand copies"},
            "gpu_launches": iters * args.steps,
            "roofline": {"bound": "tensor",
                         "kernel": "gemm_pair_kernel" if g.gemm_uses_pair(M, N, K) else "gemm_tc_kernel",
                         "achieved": achieved, "peak": tf,
                         "unit": "TFLOP/s", "frac": achieved / tf, "peak_source": kind, "traffic": None}}
    if clk:
        line["clocks"] = clk
    return line


# ------------------------------------------------------- SoVITS decoder (5)
def run_decoder(args, rank, local, world):
    import numpy as np
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    cfg = g.workloads.DECODER
    T = 500
    ws, bs = g.workloads.decoder_weights(cfg, seed=0)
    z = g.workloads.decoder_latent(T, cfg, seed=rank)  # one utterance per GPU
    dec = g.Decoder(cfg, ws, bs, max_frames=T)
    zd = torch.from_numpy(z).to(dev)
    wav = torch.empty(dec.out_len(T), device=dev)
    for _ in range(args.warmup):
        dec.forward(zd, wav)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    start.record(stream)
    for _ in range(args.steps):
        dec.forward(zd, wav)
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(start.elapsed_time(end) * 1e-3 / args.steps, world)
    # e2e: host latent in, host waveform out
    z_pin = torch.from_numpy(z).pin_memory()
    w_pin = torch.empty(wav.numel(), pin_memory=True)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        zd.copy_(z_pin, non_blocking=True)
        dec.forward(zd, wav)
        w_pin.copy_(wav, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e-3 / args.steps, world)
    flops = 2 * g.workloads.decoder_macs(cfg, T)
    launches = dec.launches()
    dec.close()
    _, tf, kind = measured_peaks()
    line = {"metric": "SoVITS decoder TFLOP/s (192x500 latent -> 320,000 samples per utterance)",
            "value": flops * world / t / 1e12, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 activations/weights, f32 accumulate and residual",
            "data": "synthetic (N(0,0.01) weights, N(0,1) latent)",
            "config": {"workload": "sovits_decoder (BASELINE configs[4])", "frames": T,
                       "samples": int(wav.numel()), "global_batch": world,
                       "parallelism": f"replicas x{world}",
                       "l2": "activations 20-40 MB per layer at the late stages, > L2 per step"},
            "e2e": {"value": flops * world / t_e2e / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": z.nbytes, "d2h_bytes_per_step": int(wav.numel()) * 4},
            "gpu_launches": launches * args.steps,
            "roofline": {"bound": "tensor", "achieved": flops / t / 1e12, "peak": tf,
                         "unit": "TFLOP/s", "frac": flops / t / 1e12 / tf, "peak_source": kind,
                         "traffic": None, "note": "whole generator; late stages are HBM-bound"}}
    if clk:
        line["clocks"] = clk
    return line


# ------------------------------------------------------ encoder prefill (4)
def run_encoder(args, rank, local, world):
    import numpy as np
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    name = args.encoder
    e = g.workloads.ENCODERS[name]
    B, T = e["batch"], e["seq"]
    m = g.workloads.encoder_model(name, seed=0)
    x = g.workloads.encoder_input(name, seed=rank)
    enc = g.Encoder(m, max_batch=B, max_seq=T)
    x0 = torch.from_numpy(x).to(dev)
    xd = torch.empty_like(x0)
    for _ in range(args.warmup):
        xd.copy_(x0)
        enc.forward(xd, B, T)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    start.record(stream)
    for _ in range(args.steps):
        xd.copy_(x0)
        enc.forward(xd, B, T)
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(start.elapsed_time(end) * 1e-3 / args.steps, world)
    # e2e: host activations in, host outputs out
    x_pin = torch.from_numpy(x).pin_memory()
    y_pin = torch.empty_like(x_pin).pin_memory()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        xd.copy_(x_pin, non_blocking=True)
        enc.forward(xd, B, T)
        y_pin.copy_(xd, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e-3 / args.steps, world)
    # the dominant kernel alone: the stack's GEMM shapes back to back
    C, F = e["hidden"], e["ffn"]
    M = B * T
    a16 = [torch.randn(M, k, device=dev).half() for k in (C, C, C, F)]
    w16 = [(torch.randn(n, k, device=dev) * 0.02).half() for n, k in ((3 * C, C), (C, C), (F, C), (C, F))]
    outs = [torch.empty(M, n, device=dev, dtype=torch.float16) for n in (3 * C, C, F, C)]
    for _ in range(3):
        for a, w_, o in zip(a16, w16, outs):
            g.gemm_ex(a, w_, c_f16=o)
    torch.cuda.synchronize(dev)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    g0.record(stream)
    for _ in range(reps):
        for a, w_, o in zip(a16, w16, outs):
            g.gemm_ex(a, w_, c_f16=o)
    g1.record(stream)
    torch.cuda.synchronize(dev)
    gemm_flops_layer = 2 * M * (3 * C * C + C * C + F * C + C * F)
    t_gemm = g0.elapsed_time(g1) * 1e-3 / reps
    launches = enc.launches()
    enc.close()
    flops = g.workloads.encoder_gemm_flops(name)
    _, tf, kind = measured_peaks()
    achieved = gemm_flops_layer / t_gemm / 1e12
    line = {"metric": f"{name} encoder prefill GEMM TFLOP/s (batch {B} x {T})",
            "value": flops * world / t / 1e12, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 operands, f32 accumulate", "data": "synthetic (N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": f"encoder_{name} (BASELINE configs[3])", "layers": e["layers"],
                       "hidden": C, "ffn": F, "global_batch": B * world, "seq_len": T,
                       "parallelism": f"replicas x{world}",
                       "flops_counted": "the stack's GEMM FLOPs; time is the whole forward",
                       "l2": "weights 0.2-0.6 GB and activations > L2 per step"},
            "e2e": {"value": flops * world / t_e2e / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x.nbytes, "d2h_bytes_per_step": x.nbytes},
            "gpu_launches": launches * args.steps,
            "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel", "achieved": achieved,
                         "peak": tf, "unit": "TFLOP/s", "frac": achieved / tf,
                         "peak_source": kind, "traffic": None,
                         "note": "the four layer GEMM shapes back to back, CUDA events"}}
    if clk:
        line["clocks"] = clk
    return line


# ------------------------------------------------- batched T2S decode (3)
def run_t2s_batch(args, rank, local, world):
    import numpy as np
    import torch

    g = __import__("__graft_entry__").package()
    g.device_init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    B, S = args.batch, 32
    m = g.workloads.t2s_model(seed=1)
    lens = g.workloads.t2s_batched_lengths(B, seed=1)
    cap = int(lens.max()) + S
    rng = np.random.default_rng(1 + rank)
    first = rng.integers(0, m["vocab"] - 1, size=B).astype(np.int32)
    hist = first[:, None].copy()
    eng = g.T2SBatch(m, cap=cap, max_batch=B, max_steps=S)
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    L, D = m["n_layers"], m["d_model"]
    for b in range(B):  # KV prefix N(0,1) fp16, drawn on the device
        k = torch.randn(L, int(lens[b]), D, generator=gen, device=dev).half()
        v = torch.randn(L, int(lens[b]), D, generator=gen, device=dev).half()
        eng.load_kv(b, k, v, int(lens[b]))
    torch.cuda.synchronize(dev)

    def one():
        eng.begin(lens, lens, first, hist)
        eng.run(S, use_graph=True)

    eng.begin(lens, lens, first, hist)
    eng.run(S, use_graph=False)  # eager once (attributes, descriptors), then graphs
    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    clocks = ClockSampler()
    barrier(world)
    clocks.start()
    for i in range(args.steps):
        eng.begin(lens, lens, first, hist)
        ev[i][0].record(stream)
        eng.run(S, use_graph=True)
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    t = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) * 1e-3 / args.steps, world)
    # e2e: host token ids in, host tokens out (begin copies the per-utterance state)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.begin(lens, lens, first, hist)
        eng.run(S, use_graph=True)
        toks, _ = eng.read(S)
    t_e2e = max_over_ranks(time.perf_counter() - t0, world) / args.steps
    launches = eng.launches_per_step()
    eng.close()
    w_bytes = L * (3 * D * D + D * D + 2 * m["ffn"] * D) * 2 + m["vocab"] * D * 2
    kv = L * 2 * D * 2
    alg = sum(w_bytes + kv * int(np.sum(lens + s + 1)) + kv * B for s in range(S))
    hbm, _, kind = measured_peaks()
    tokens = B * S
    line = {"metric": f"batched T2S decode tokens/s ({B} utterances per GPU)",
            "value": tokens * world / t, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 operands, f32 accumulate",
            "data": "synthetic (N(0,0.02) weights, N(0,1) KV, lengths U{64..1024} seed 1)",
            "config": {"workload": "t2s_decode_b64 (BASELINE configs[2])", "batch": B,
                       "decode_steps_per_step": S, "mean_kv_len": float(lens.mean()),
                       "global_batch": B * world, "parallelism": f"replicas x{world}",
                       "l2": "1.9 GB of weights + KV streamed per decode step"},
            "e2e": {"value": tokens * world / t_e2e, "unit": "tokens/s",
                    "h2d_bytes_per_step": int(lens.nbytes * 2 + first.nbytes + hist.nbytes),
                    "d2h_bytes_per_step": tokens * 8, "timing": "host wall clock"},
            "gpu_launches": launches * S * args.steps,
            "roofline": {"bound": "hbm", "kernel": "decode step (CUDA graph)",
                         "achieved": alg / t / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": alg / t / 1e9 / hbm, "peak_source": kind, "traffic": None,
                         "algorithmic_bytes_per_step": alg}}
    if clk:
        line["clocks"] = clk
    return line


WORKLOADS = {"t2s_decode_b1": run_t2s, "gemm_ffn_up": run_gemm1, "sovits_decoder": run_decoder,
             "gemv_t2s": run_gemv_t2s, "encoder": run_encoder, "hubert_front": run_engine,
             "sovits_latent": run_engine, "sv": run_engine, "t2s_decode_b64": run_t2s_batch, "gemm": run_gemm_shape}


def run_reference(args, rank, world):
    """The reference's CPU arithmetic (the oracle restatement) on the host
    cores: each step is one bounded sample of the workload, timed whole; the
    line's value is the median step in the workload's unit."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    fn, units, desc = cpu_sampler(args, threads)
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    meta = workload_meta(args, 1)
    cb = cpu_result(args, units, desc, times, threads)
    return {"metric": meta["metric"], "value": cb["value"], "unit": meta["unit"],
            "impl": "reference", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(times) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": meta["dtype"], "data": meta["data"],
            "config": meta["config"], "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": meta["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    global T2S_STEPS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="gsvk", choices=["gsvk", "reference"])
    ap.add_argument("--workload", default="t2s_decode_b1", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip the profiler-based kernel count (e.g. under ncu)")
    ap.add_argument("--encoder", default="bert", choices=["bert", "hubert"])
    ap.add_argument("--gemm-shape", default="4096,4096,1024",
                    help="M,N,K of the gemm workload")
    ap.add_argument("--batch", type=int, default=64,
                    help="utterances of the t2s_decode_b64 workload (64 = BASELINE config 3)")
    ap.add_argument("--decode-kernel", type=int, default=0,
                    help="t2s_decode_b1 decode kernel (gsvk_t2s_set_decode_kernel; 0 = default)")
    ap.add_argument("--decode-steps", type=int, default=T2S_STEPS,
                    help="tokens per utterance (default 500; smaller only for profiling captures)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    T2S_STEPS = args.decode_steps
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    rank, local, world = dist_setup(args.gpus)
    try:
        line = WORKLOADS[args.workload](args, rank, local, world)
    finally:
        pass
    if rank == 0:
        # every arm prints the same metric, unit and config for the workload
        meta = workload_meta(args, world)
        extra = {k: v for k, v in line.get("config", {}).items() if k not in meta["config"]}
        line.update(metric=meta["metric"], unit=meta["unit"], config=meta["config"])
        line.setdefault("dtype", meta["dtype"])
        line.setdefault("data", meta["data"])
        if extra:
            line["run"] = extra
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_measure(args)
    dist_close(world)
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
