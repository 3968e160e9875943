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


HUBERT_FRONT = dict(conv_dim=(512,) * 7, conv_kernel=(10, 3, 3, 3, 3, 2, 2),
                    conv_stride=(5, 2, 2, 2, 2, 2, 2), hidden=768, pos_k=128, pos_groups=16,
                    ln_eps=1e-5)


def hubert_front_model(seed=0, cfg=HUBERT_FRONT) -> dict:
    """HuBERT feature front-end weights (hubert.cpp:93-160 layouts): conv
    weights fp16 [512][in][k] ~ N(0, 1/fan_in), GroupNorm / LayerNorm gains
    1+N(0,0.05) and biases N(0,0.02), projection fp16 [768][512] N(0,0.02)
    and bias, positional conv fp32 [768][48][128] N(0, 1/fan_in) and bias."""
    rng = np.random.default_rng(seed)
    m = dict(cfg)
    m["conv_w"] = []
    ci = 1
    for co, k in zip(cfg["conv_dim"], cfg["conv_kernel"]):
        m["conv_w"].append(_f16(_normal(rng, (co, ci, k), 1.0 / np.sqrt(ci * k))))
        ci = co
    C0, C6, H = cfg["conv_dim"][0], cfg["conv_dim"][6], cfg["hidden"]
    cg = H // cfg["pos_groups"]
    m["gn_g"] = (1.0 + _normal(rng, (C0,), 0.05)).astype(np.float32)
    m["gn_b"] = _normal(rng, (C0,), 0.02)
    m["proj_ln_g"] = (1.0 + _normal(rng, (C6,), 0.05)).astype(np.float32)
    m["proj_ln_b"] = _normal(rng, (C6,), 0.02)
    m["proj_w"] = _f16(_normal(rng, (H, C6), 0.02))
    m["proj_b"] = _normal(rng, (H,), 0.02)
    m["pos_w"] = _normal(rng, (H, cg, cfg["pos_k"]), 1.0 / np.sqrt(cg * cfg["pos_k"]))
    m["pos_b"] = _normal(rng, (H,), 0.02)
    m["enc_ln_g"] = (1.0 + _normal(rng, (H,), 0.05)).astype(np.float32)
    m["enc_ln_b"] = _normal(rng, (H,), 0.02)
    return m


def hubert_waveform(n=16000, seed=0):
    """A waveform stand-in ~ N(0, 0.1) (the reference feeds 16 kHz audio)."""
    return _normal(np.random.default_rng(seed + 7000), (n,), 0.1)


SOVITS_LATENT = dict(ssl_dim=768, hidden=192, filter=768, heads=2, kernel=3, window=4,
                     layers_ssl=3, layers_text=6, layers_2=3, mrte_hidden=512, mrte_heads=4,
                     gin=1024, flows=4, wn_layers=4, wn_kernel=5, noise_scale=0.5,
                     n_symbols=732, codebook=1024)


def sovits_latent_model(seed=0, cfg=SOVITS_LATENT) -> dict:
    """The SoVITS latent path's tensors under their .gsv names (enc_p.hpp,
    enc_p_parts.hpp, mha.hpp, flow.hpp, quantizer.hpp): conv weights fp16
    [out][in][k] ~ N(0, 1/fan_in), biases N(0, 0.02), LayerNorm gains
    1+N(0,0.05), relative tables N(0, dk^-1/2) [1][2W+1][dk], text embedding
    N(0, hidden^-1/2), codebook N(0,1) - the torch initialisers' scales."""
    rng = np.random.default_rng(seed)
    c = dict(cfg)
    C, H, F, K = c["hidden"], c["heads"], c["filter"], c["kernel"]
    t = {}

    def conv(name, co, ci, k, wscale=1.0):
        t[name + ".weight"] = _f16(_normal(rng, (co, ci, k), wscale / np.sqrt(ci * k)))
        t[name + ".bias"] = _normal(rng, (co,), 0.02)

    def mha(p, ch, heads, rel):
        for n in ("q", "k", "v", "o"):
            conv(f"{p}.conv_{n}", ch, ch, 1)
        if rel:
            dk = ch // heads
            for n in ("k", "v"):
                t[f"{p}.emb_rel_{n}"] = _normal(rng, (1, 2 * c["window"] + 1, dk), dk ** -0.5)

    def encoder(p, nl):
        for i in range(nl):
            mha(f"{p}.attn_layers.{i}", C, H, True)
            for j in (1, 2):
                t[f"{p}.norm_layers_{j}.{i}.gamma"] = (1 + _normal(rng, (C,), 0.05)).astype(np.float32)
                t[f"{p}.norm_layers_{j}.{i}.beta"] = _normal(rng, (C,), 0.02)
            conv(f"{p}.ffn_layers.{i}.conv_1", F, C, K)
            conv(f"{p}.ffn_layers.{i}.conv_2", C, F, K)

    t["quantizer.vq.layers.0._codebook.embed"] = _normal(rng, (c["codebook"], c["ssl_dim"]), 1.0)
    conv("enc_p.ssl_proj", C, c["ssl_dim"], 1)
    encoder("enc_p.encoder_ssl", c["layers_ssl"])
    encoder("enc_p.encoder_text", c["layers_text"])
    encoder("enc_p.encoder2", c["layers_2"])
    t["enc_p.text_embedding.weight"] = _normal(rng, (c["n_symbols"], C), C ** -0.5)
    MH = c["mrte_hidden"]
    mha("enc_p.mrte.cross_attention", MH, c["mrte_heads"], False)
    conv("enc_p.mrte.c_pre", MH, C, 1)
    conv("enc_p.mrte.text_pre", MH, C, 1)
    conv("enc_p.mrte.c_post", C, MH, 1)
    conv("enc_p.proj", 2 * C, C, 1)
    nl = c["wn_layers"]
    for f in range(c["flows"]):
        p = f"flow.flows.{2 * f}"
        conv(p + ".pre", C, C // 2, 1)
        conv(p + ".enc.cond_layer", 2 * C * nl, c["gin"], 1)
        for i in range(nl):
            conv(f"{p}.enc.in_layers.{i}", 2 * C, C, c["wn_kernel"])
            conv(f"{p}.enc.res_skip_layers.{i}", 2 * C if i + 1 < nl else C, C, 1)
        conv(p + ".post", C // 2, C, 1, wscale=0.5)
    c["tensors"] = t
    return c


def sovits_latent_inputs(n_codes, n_phones, cfg=SOVITS_LATENT, seed=0, noise=True):
    """codes U[0, codebook), phones U[0, n_symbols), ge N(0,1) [gin],
    ge_text N(0,1) [mrte_hidden], noise N(0,1) [hidden][2 n_codes]."""
    rng = np.random.default_rng(seed + 9000)
    codes = rng.integers(0, cfg["codebook"], n_codes).astype(np.int64)
    phones = rng.integers(0, cfg["n_symbols"], n_phones).astype(np.int64)
    ge = _normal(rng, (cfg["gin"],), 1.0)
    ge_text = _normal(rng, (cfg["mrte_hidden"],), 1.0)
    nz = _normal(rng, (cfg["hidden"], 2 * n_codes), 1.0) if noise else None
    return codes, phones, ge, ge_text, nz


SV_STAGES = ((3, 1, False), (4, 2, False), (6, 2, True), (3, 2, True))  # blocks, stride, AFF


def sv_model(seed=0, m_ch=64, base_width=24, scale=4, expansion=4) -> dict:
    """ERes2NetV2 w24 s4 e4 tensors under their .gsv names (sv.cpp:660-760):
    convs fp16 [out][in][kh][kw] ~ N(0, 2/fan_in) (He; the residual-branch
    conv3 and the shortcuts x0.25, which keeps relu20 mostly unsaturated),
    the stem conv fp32, BatchNorm gamma 1+N(0,0.1), beta N(0,0.1), running
    mean N(0,0.1), running var U(0.5,1.5); the AFF second convs fp32 only
    (the reference rounds those once)."""
    rng = np.random.default_rng(seed)
    t = {}

    def conv(name, co, ci, k, gain=1.0, f32=False):
        w = _normal(rng, (co, ci, k, k), gain * np.sqrt(2.0 / (ci * k * k)))
        t[name] = w if f32 else _f16(w)

    def bn(p, c):
        t[p + ".weight"] = (1 + _normal(rng, (c,), 0.1)).astype(np.float32)
        t[p + ".bias"] = _normal(rng, (c,), 0.1)
        t[p + ".running_mean"] = _normal(rng, (c,), 0.1)
        t[p + ".running_var"] = rng.uniform(0.5, 1.5, c).astype(np.float32)

    def aff(p, ch, r=4):
        inter = ch // r
        conv(p + "0.weight", inter, 2 * ch, 1)
        t[p + "0.bias"] = _normal(rng, (inter,), 0.1)
        bn(p + "1", inter)
        conv(p + "3.weight", ch, inter, 1, gain=0.5, f32=True)
        t[p + "3.bias"] = _normal(rng, (ch,), 0.1)
        bn(p + "4", ch)

    conv("conv1.weight", m_ch, 1, 3, f32=True)
    bn("bn1", m_ch)
    c_in = m_ch
    for l, (blocks, stride, with_aff) in enumerate(SV_STAGES, 1):
        planes = m_ch * 2 ** (l - 1)
        width = planes * base_width // 64
        exp = planes * expansion
        for i in range(blocks):
            p = f"layer{l}.{i}."
            conv(p + "conv1.weight", width * scale, c_in, 1)
            bn(p + "bn1", width * scale)
            for j in range(scale):
                conv(p + f"convs.{j}.weight", width, width, 3)
                bn(p + f"bns.{j}", width)
            conv(p + "conv3.weight", exp, width * scale, 1, gain=0.25)
            bn(p + "bn3", exp)
            if with_aff:
                for j in range(scale - 1):
                    aff(p + f"fuse_models.{j}.local_att.", width)
            if i == 0 and (stride != 1 or c_in != exp):
                conv(p + "shortcut.0.weight", exp, c_in, 1, gain=0.25)
                bn(p + "shortcut.1", exp)
            c_in = exp
        if l == 3:
            c3 = exp
    conv("layer3_ds.weight", c_in, c3, 3, gain=0.5)
    aff("fuse34.local_att.", c_in)
    return {"tensors": t, "m_ch": m_ch, "emb_channels": c_in}


def sv_fbank(frames=64, n_mels=80, seed=0):
    """A log-mel stand-in: N(0,1) [frames][n_mels] (fbank.cpp output shape)."""
    return _normal(np.random.default_rng(seed + 11000), (frames, n_mels), 1.0)


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
