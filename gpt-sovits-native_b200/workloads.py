"""Seeded synthetic inputs for the five benchmark configurations.

The reference names no public dataset; every tensor here is drawn from a
seeded numpy PCG64 generator with the shapes and value distributions the
configurations state, so the CUDA path, the CPU oracle and the CPU baseline
all see bit-identical inputs.  fp16 tensors are returned as uint16 bit
patterns (IEEE binary16, round-to-nearest-even from fp32).
"""
from __future__ import annotations

import numpy as np


def _f16(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16).view(np.uint16))


def _normal(rng, shape, std):
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)


# ------------------------------------------------------------------ config 1
def gemm_ffn_up(M=128, N=2048, K=512, seed=0):
    """Y = ReLU(X W^T + b): X U(-1,1) fp16, W N(0,0.02) fp16, b N(0,0.01) fp32."""
    rng = np.random.default_rng(seed)
    x = _f16(rng.uniform(-1.0, 1.0, size=(M, K)).astype(np.float32))
    w = _f16(_normal(rng, (N, K), 0.02))
    b = _normal(rng, (N,), 0.01)
    return x, w, b


# -------------------------------------------------------------- configs 2, 3
T2S_SHAPE = dict(n_layers=24, d_model=512, n_heads=16, ffn=2048, vocab=1025)


def t2s_model(n_layers=24, d_model=512, n_heads=16, ffn=2048, vocab=1025, seed=0):
    """T2S transformer weights (post-LN, fused QKV, ReLU FFN, logits head
    without bias).  Linear weights N(0,0.02) fp16, biases N(0,0.02) fp32,
    LayerNorm gain 1+N(0,0.05) and bias N(0,0.02), audio embedding N(0,0.02)."""
    rng = np.random.default_rng(seed)
    L, D, F, V = n_layers, d_model, ffn, vocab
    m = dict(n_layers=L, d_model=D, n_heads=n_heads, ffn=F, vocab=V, ln_eps=1e-5,
             alpha_audio=1.0)
    m["wqkv"] = _f16(_normal(rng, (L, 3 * D, D), 0.02))
    m["bqkv"] = _normal(rng, (L, 3 * D), 0.02)
    m["wout"] = _f16(_normal(rng, (L, D, D), 0.02))
    m["bout"] = _normal(rng, (L, D), 0.02)
    m["w1"] = _f16(_normal(rng, (L, F, D), 0.02))
    m["b1"] = _normal(rng, (L, F), 0.02)
    m["w2"] = _f16(_normal(rng, (L, D, F), 0.02))
    m["b2"] = _normal(rng, (L, D), 0.02)
    m["n1g"] = (1.0 + _normal(rng, (L, D), 0.05)).astype(np.float32)
    m["n1b"] = _normal(rng, (L, D), 0.02)
    m["n2g"] = (1.0 + _normal(rng, (L, D), 0.05)).astype(np.float32)
    m["n2b"] = _normal(rng, (L, D), 0.02)
    m["wpred"] = _f16(_normal(rng, (V, D), 0.02))
    m["audio_emb"] = _f16(_normal(rng, (V, D), 0.02))
    return m


def t2s_kv_prefix(model: dict, cap: int, prefix: int, seed=0):
    """KV caches [L, cap, D] fp16 with slots [0, prefix) ~ N(0,1), rest 0."""
    rng = np.random.default_rng(seed + 1000)
    L, D = model["n_layers"], model["d_model"]
    k = np.zeros((L, cap, D), np.uint16)
    v = np.zeros((L, cap, D), np.uint16)
    k[:, :prefix] = _f16(_normal(rng, (L, prefix, D), 1.0))
    v[:, :prefix] = _f16(_normal(rng, (L, prefix, D), 1.0))
    return k, v


def t2s_prompt(P=64, vocab=1025, seed=0):
    """Prompt semantic ids uniform in [0, vocab-1) (EOS excluded)."""
    rng = np.random.default_rng(seed + 2000)
    return rng.integers(0, vocab - 1, size=P).astype(np.int32)


def t2s_decode_b1(seed=0, prefix=256, P=64, steps=500, **shape):
    """Config 2: batch-1 decode, KV prefix of 256 slots, 64-token prompt."""
    s = dict(T2S_SHAPE)
    s.update(shape)
    m = t2s_model(seed=seed, **s)
    cap = prefix + P + steps
    k, v = t2s_kv_prefix(m, cap, prefix, seed=seed)
    return m, k, v, t2s_prompt(P, m["vocab"], seed=seed)


def t2s_batched_lengths(B=64, lo=64, hi=1024, seed=1):
    """Config 3: per-utterance KV lengths uniform in [lo, hi]."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=B).astype(np.int32)


# ------------------------------------------------------------------ config 4
ENCODERS = {
    "bert": dict(layers=24, hidden=1024, heads=16, ffn=4096, batch=32, seq=128, eps=1e-12),
    "hubert": dict(layers=12, hidden=768, heads=12, ffn=3072, batch=32, seq=250, eps=1e-5),
}


def encoder_model(name: str, layers=None, seed=0) -> dict:
    """Encoder weights in the oracle / C-ABI layout: q, k, v rows fused as
    [L][3C][C]; N(0,0.02) fp16 matrices, N(0,0.02) fp32 biases, LayerNorm gain
    1+N(0,0.05), bias N(0,0.02)."""
    e = ENCODERS[name]
    rng = np.random.default_rng(seed)
    L = layers or e["layers"]
    C, F = e["hidden"], e["ffn"]
    m = dict(layers=L, hidden=C, heads=e["heads"], ffn=F, eps=e["eps"])
    m["wqkv"] = _f16(_normal(rng, (L, 3 * C, C), 0.02))
    m["bqkv"] = _normal(rng, (L, 3 * C), 0.02)
    m["wo"] = _f16(_normal(rng, (L, C, C), 0.02))
    m["bo"] = _normal(rng, (L, C), 0.02)
    m["ln1g"] = (1.0 + _normal(rng, (L, C), 0.05)).astype(np.float32)
    m["ln1b"] = _normal(rng, (L, C), 0.02)
    m["wi"] = _f16(_normal(rng, (L, F, C), 0.02))
    m["bi"] = _normal(rng, (L, F), 0.02)
    m["wf"] = _f16(_normal(rng, (L, C, F), 0.02))
    m["bf"] = _normal(rng, (L, C), 0.02)
    m["ln2g"] = (1.0 + _normal(rng, (L, C), 0.05)).astype(np.float32)
    m["ln2b"] = _normal(rng, (L, C), 0.02)
    return m


def encoder_input(name: str, batch=None, seq=None, seed=0) -> np.ndarray:
    """Activations N(0,1) fp32 [batch*seq, hidden]."""
    e = ENCODERS[name]
    rng = np.random.default_rng(seed + 5000)
    return _normal(rng, ((batch or e["batch"]) * (seq or e["seq"]), e["hidden"]), 1.0)


def encoder_gemm_flops(name: str) -> int:
    e = ENCODERS[name]
    M, H, Fd = e["batch"] * e["seq"], e["hidden"], e["ffn"]
    per_layer = 2 * M * (H * 3 * H + H * H + H * Fd + Fd * H)
    return e["layers"] * per_layer


# ------------------------------------------------------------------ config 5
DECODER = dict(n_stages=5, in_ch=192, ch0=512, up_rate=(10, 8, 2, 2, 2), up_k=(16, 16, 8, 2, 2),
               res_k=(3, 7, 11), res_dil=(1, 3, 5), conv_pre_k=7, conv_post_k=7,
               lrelu_slope=0.1, post_slope=0.01)
# The reference v2ProPlus generator (dec.hpp:55-76): second parity case.
DECODER_REF = dict(DECODER, ch0=768, up_k=(20, 16, 8, 2, 2))


def decoder_weights(cfg=DECODER, seed=0, std=0.01):
    """Weights in the order documented in oracle.h (conv_pre, per stage: ups,
    3 resblocks x 3 (convs1, convs2) pairs; conv_post without bias), torch
    layouts: Conv1d [Co,Ci,k], ConvTranspose1d [Ci,Co,k]."""
    rng = np.random.default_rng(seed)
    ws, bs = [], []
    C = cfg["ch0"]
    ws.append(_f16(_normal(rng, (C, cfg["in_ch"], cfg["conv_pre_k"]), std)))
    bs.append(_normal(rng, (C,), std))
    for s in range(cfg["n_stages"]):
        Cn = C // 2
        ws.append(_f16(_normal(rng, (C, Cn, cfg["up_k"][s]), std)))
        bs.append(_normal(rng, (Cn,), std))
        for j in range(3):
            for p in range(3):
                for _ in range(2):
                    ws.append(_f16(_normal(rng, (Cn, Cn, cfg["res_k"][j]), std)))
                    bs.append(_normal(rng, (Cn,), std))
        C = Cn
    ws.append(_f16(_normal(rng, (1, C, cfg["conv_post_k"]), std)))
    bs.append(None)
    return ws, bs


def decoder_latent(T=500, cfg=DECODER, seed=0):
    rng = np.random.default_rng(seed + 3000)
    return _normal(rng, (cfg["in_ch"], T), 1.0)


def decoder_macs(cfg=DECODER, T=500) -> int:
    """Multiply-accumulates of one generator pass (conv_pre, ConvT, resblocks,
    conv_post), counted as Co*Ci*k per output sample."""
    C, L = cfg["ch0"], T
    macs = C * cfg["in_ch"] * cfg["conv_pre_k"] * L
    for s in range(cfg["n_stages"]):
        Cn, Ln = C // 2, L * cfg["up_rate"][s]
        macs += C * Cn * cfg["up_k"][s] * L  # ConvT: each input sample meets k taps
        for j in range(3):
            macs += 6 * Cn * Cn * cfg["res_k"][j] * Ln
        C, L = Cn, Ln
    macs += C * cfg["conv_post_k"] * L
    return macs
