"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker, and by bench.py's CPU-baseline leg.  The CUDA product path never
imports this module.

The C sources (oracle.cpp) restate the reference project's src/kern arithmetic;
each function there cites the reference file:line it follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_char, c_double, c_float, c_int, c_size_t, c_uint16, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

ACT_NONE, ACT_RELU, ACT_GELU_ERF, ACT_LEAKY = 0, 1, 2, 3


def build(force: bool = False) -> str:
    """Compile liboracle.so with the Makefile next to this file."""
    src = os.path.join(_HERE, "oracle.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


class T2SDims(ctypes.Structure):
    _fields_ = [("n_layers", c_int), ("d_model", c_int), ("n_heads", c_int), ("ffn", c_int),
                ("vocab", c_int), ("ln_eps", c_float), ("alpha_audio", c_float)]


class T2SWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in (
        "wqkv", "bqkv", "wout", "bout", "w1", "b1", "w2", "b2",
        "n1g", "n1b", "n2g", "n2b", "wpred", "audio_emb")]


class EncoderDims(ctypes.Structure):
    _fields_ = [("layers", c_int), ("hidden", c_int), ("heads", c_int), ("ffn", c_int),
                ("eps", c_double)]


class EncoderWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("wqkv", "bqkv", "wo", "bo", "ln1g", "ln1b", "wi", "bi",
                                        "wf", "bf", "ln2g", "ln2b")]


class DecoderCfg(ctypes.Structure):
    _fields_ = [("n_stages", c_int), ("in_ch", c_int), ("ch0", c_int), ("conv_pre_k", c_int),
                ("conv_post_k", c_int), ("up_rate", c_int * 8), ("up_k", c_int * 8),
                ("res_k", c_int * 3), ("res_dil", c_int * 3), ("lrelu_slope", c_float),
                ("post_slope", c_float)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, sz = c_void_p, c_size_t
        sigs = {
            "ora_set_threads": (None, [c_int]),
            "ora_get_threads": (c_int, []),
            "ora_f32_to_f16": (None, [vp, vp, sz]),
            "ora_f16_to_f32": (None, [vp, vp, sz]),
            "ora_gemv_f16w_f32acc_ref": (None, [vp, vp, vp, sz, sz]),
            "ora_gemv_f16w_f32acc": (None, [vp, vp, vp, sz, sz]),
            "ora_gemv_f16x_fmlal": (None, [vp, vp, vp, sz, sz]),
            "ora_gemm_f16x_fmlal": (None, [vp, vp, vp, sz, sz, sz]),
            "ora_sgemm": (None, [c_char, c_char, c_int, c_int, c_int, c_float, vp, c_int, vp,
                                 c_int, c_float, vp, c_int]),
            "ora_linear_f16": (None, [vp, sz, sz, vp, sz, vp, c_int, c_float, vp]),
            "ora_layernorm": (None, [vp, vp, vp, vp, sz, c_double]),
            "ora_rmsnorm": (None, [vp, vp, vp, sz, c_double]),
            "ora_softmax": (None, [vp, vp, sz]),
            "ora_relu": (None, [vp, vp, sz]),
            "ora_silu": (None, [vp, vp, sz]),
            "ora_gelu_erf": (None, [vp, vp, sz]),
            "ora_leaky_relu": (None, [vp, vp, sz, c_float]),
            "ora_conv1d": (None, [vp, sz, sz, vp, vp, sz, sz, sz, c_int, vp]),
            "ora_convt1d": (None, [vp, sz, sz, vp, vp, sz, sz, sz, c_int, vp]),
            "ora_decoder_out_len": (sz, [vp, sz]),
            "ora_decoder_forward": (None, [vp, vp, vp, vp, sz, c_int, vp]),
            "ora_t2s_pe_row": (None, [c_int, sz, vp]),
            "ora_t2s_decode_layer": (None, [vp, vp, c_int, vp, sz, vp, vp]),
            "ora_t2s_prefill_layer": (None, [vp, vp, c_int, vp, sz, sz, sz, vp, vp]),
            "ora_t2s_greedy_sample": (c_int, [vp, c_int, vp, sz, c_int, vp]),
            "ora_attention_decode": (None, [vp, vp, vp, sz, sz, sz, sz, c_float, vp]),
            "ora_encoder_layer": (None, [vp, vp, c_int, vp, c_int, c_int, vp]),
            "ora_t2s_generate": (c_int, [vp, vp, vp, vp, sz, sz, vp, sz, sz, c_int, vp, vp, vp]),
            "ora_t2s_decode_layer_literal": (None, [vp, vp, c_int, vp, sz, vp, vp]),
            "ora_t2s_generate_sampled": (c_int, [vp, vp, vp, vp, sz, sz, vp, sz, sz, c_int, vp,
                                                 vp, vp]),
            "ora_sovits_latent": (c_int, [vp, vp, sz, vp, sz, vp, sz, vp, vp, vp, vp, vp, vp]),
            "ora_sv_forward": (sz, [vp, sz, vp, sz, c_int, vp]),
            "ora_sv_conv2d_f16": (None, [vp, c_int, c_int, c_int, vp, c_int, c_int, c_int, c_int,
                                         c_int, vp]),
            "ora_hubert_front_frames": (sz, [vp, sz]),
            "ora_hubert_front": (None, [vp, vp, vp, sz, vp]),
            "ora_t2s_generate_ex": (c_int, [vp, vp, vp, vp, sz, sz, vp, sz, sz, c_int, c_int, vp,
                                            vp, vp]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().ora_set_threads(int(n))


def get_threads() -> int:
    return lib().ora_get_threads()


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ora_f32_to_f16(_p(x), _p(out), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().ora_f16_to_f32(_p(h), _p(out), h.size)
    return out


def gemv_f16w_f32acc(w: np.ndarray, x: np.ndarray, ref: bool = False) -> np.ndarray:
    out_, in_ = w.shape
    y = np.empty(out_, dtype=np.float32)
    fn = lib().ora_gemv_f16w_f32acc_ref if ref else lib().ora_gemv_f16w_f32acc
    fn(_p(w), _p(np.ascontiguousarray(x, np.float32)), _p(y), out_, in_)
    return y


def gemv_f16x_fmlal(w: np.ndarray, xh: np.ndarray) -> np.ndarray:
    out_, in_ = w.shape
    y = np.empty(out_, dtype=np.float32)
    lib().ora_gemv_f16x_fmlal(_p(w), _p(np.ascontiguousarray(xh, np.uint16)), _p(y), out_, in_)
    return y


def gemm_f16x_fmlal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    M, K = a.shape
    N, K2 = b.shape
    assert K == K2
    c = np.empty((M, N), dtype=np.float32)
    lib().ora_gemm_f16x_fmlal(_p(a), _p(b), _p(c), M, N, K)
    return c


def sgemm(ta: str, tb: str, M: int, N: int, K: int, alpha: float, A, lda: int, B, ldb: int,
          beta: float, C, ldc: int) -> None:
    lib().ora_sgemm(ta.encode(), tb.encode(), M, N, K, alpha, _p(A), lda, _p(B), ldb, beta,
                    _p(C), ldc)


def linear_f16(x: np.ndarray, w: np.ndarray, bias=None, act: int = ACT_NONE,
               slope: float = 0.0) -> np.ndarray:
    T, in_ = x.shape
    out_ = w.shape[0]
    y = np.empty((T, out_), dtype=np.float32)
    lib().ora_linear_f16(_p(np.ascontiguousarray(x, np.float32)), T, in_, _p(w), out_, _p(bias),
                         act, slope, _p(y))
    return y


def layernorm(x: np.ndarray, g: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    n = x.shape[-1]
    for r in range(x.size // n):
        lib().ora_layernorm(x.ctypes.data + 4 * r * n, _p(g), _p(b), y.ctypes.data + 4 * r * n,
                            n, eps)
    return y


def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    n = x.shape[-1]
    for r in range(x.size // n):
        lib().ora_rmsnorm(x.ctypes.data + 4 * r * n, _p(g), y.ctypes.data + 4 * r * n, n, eps)
    return y


def softmax_rows(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    n = x.shape[-1]
    for r in range(x.size // n):
        lib().ora_softmax(x.ctypes.data + 4 * r * n, y.ctypes.data + 4 * r * n, n)
    return y


def _elementwise(name: str, x: np.ndarray, *extra) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    getattr(lib(), name)(_p(x), _p(y), x.size, *extra)
    return y


def relu(x):
    return _elementwise("ora_relu", x)


def silu(x):
    return _elementwise("ora_silu", x)


def gelu_erf(x):
    return _elementwise("ora_gelu_erf", x)


def leaky_relu(x, slope: float):
    return _elementwise("ora_leaky_relu", x, slope)


def conv1d(x: np.ndarray, w: np.ndarray, bias, dil: int = 1, round_in: bool = True) -> np.ndarray:
    """x [Ci,T] fp32, w [Co,Ci,k] fp16 bits (torch layout) -> y [Co,T]."""
    Ci, T = x.shape
    Co, Ci2, k = w.shape
    assert Ci == Ci2
    y = np.empty((Co, T), dtype=np.float32)
    lib().ora_conv1d(_p(np.ascontiguousarray(x, np.float32)), Ci, T, _p(w), _p(bias), Co, k, dil,
                     int(round_in), _p(y))
    return y


def convt1d(x: np.ndarray, w: np.ndarray, bias, u: int, round_in: bool = True) -> np.ndarray:
    """x [Ci,T] fp32, w [Ci,Co,k] fp16 bits (torch layout) -> y [Co,T*u]."""
    Ci, T = x.shape
    Ci2, Co, k = w.shape
    assert Ci == Ci2
    y = np.empty((Co, T * u), dtype=np.float32)
    lib().ora_convt1d(_p(np.ascontiguousarray(x, np.float32)), Ci, T, _p(w), _p(bias), Co, k, u,
                      int(round_in), _p(y))
    return y


def decoder_cfg(n_stages=5, in_ch=192, ch0=512, up_rate=(10, 8, 2, 2, 2), up_k=(16, 16, 8, 2, 2),
                res_k=(3, 7, 11), res_dil=(1, 3, 5), conv_pre_k=7, conv_post_k=7,
                lrelu_slope=0.1, post_slope=0.01) -> DecoderCfg:
    c = DecoderCfg()
    c.n_stages, c.in_ch, c.ch0 = n_stages, in_ch, ch0
    c.conv_pre_k, c.conv_post_k = conv_pre_k, conv_post_k
    for i in range(n_stages):
        c.up_rate[i] = up_rate[i]
        c.up_k[i] = up_k[i]
    for i in range(3):
        c.res_k[i] = res_k[i]
        c.res_dil[i] = res_dil[i]
    c.lrelu_slope, c.post_slope = lrelu_slope, post_slope
    return c


def decoder_forward(cfg: DecoderCfg, ws: list, bs: list, z: np.ndarray,
                    round_in: bool = True) -> np.ndarray:
    T = z.shape[1]
    n_out = lib().ora_decoder_out_len(ctypes.byref(cfg), T)
    wav = np.empty(n_out, dtype=np.float32)
    wp = (c_void_p * len(ws))(*[_p(w) for w in ws])
    bp = (c_void_p * len(bs))(*[_p(b) for b in bs])
    lib().ora_decoder_forward(ctypes.byref(cfg), wp, bp, _p(np.ascontiguousarray(z, np.float32)),
                              T, int(round_in), _p(wav))
    return wav


def t2s_structs(model: dict):
    """model: dict of numpy arrays (see tests/golden workload generator)."""
    d = T2SDims(model["n_layers"], model["d_model"], model["n_heads"], model["ffn"],
                model["vocab"], model["ln_eps"], model["alpha_audio"])
    w = T2SWeights(*[_p(model[n]) for n in (
        "wqkv", "bqkv", "wout", "bout", "w1", "b1", "w2", "b2",
        "n1g", "n1b", "n2g", "n2b", "wpred", "audio_emb")])
    return d, w


def t2s_pe_row(d_model: int, pos: int) -> np.ndarray:
    pe = np.empty(d_model, dtype=np.float32)
    lib().ora_t2s_pe_row(d_model, pos, _p(pe))
    return pe


def t2s_decode_layer(model: dict, layer: int, x: np.ndarray, pos: int, kc: np.ndarray,
                     vc: np.ndarray) -> None:
    d, w = t2s_structs(model)
    lib().ora_t2s_decode_layer(ctypes.byref(d), ctypes.byref(w), layer, _p(x), pos, _p(kc), _p(vc))


def t2s_prefill_layer(model: dict, layer: int, x: np.ndarray, pos: int, text_len: int,
                      kc: np.ndarray, vc: np.ndarray) -> None:
    d, w = t2s_structs(model)
    lib().ora_t2s_prefill_layer(ctypes.byref(d), ctypes.byref(w), layer, _p(x), x.shape[0], pos,
                                text_len, _p(kc), _p(vc))


def attention_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, length: int, n_heads: int,
                     head_dim: int, scale: float) -> np.ndarray:
    """q [H*HD] fp32; kc/vc [slots, row_stride] fp16 bits."""
    out = np.zeros(n_heads * head_dim, np.float32)
    lib().ora_attention_decode(_p(np.ascontiguousarray(q, np.float32)), _p(kc), _p(vc), length,
                               n_heads, head_dim, kc.shape[1], scale, _p(out))
    return out


def t2s_greedy_sample(logits: np.ndarray, history: np.ndarray, eos_allowed: bool):
    raw = c_int(-1)
    h = np.ascontiguousarray(history, np.int32)
    s = lib().ora_t2s_greedy_sample(_p(logits), logits.size, _p(h), h.size, int(eos_allowed),
                                    ctypes.byref(raw))
    return s, raw.value


def t2s_generate(model: dict, kcache: np.ndarray, vcache: np.ndarray, prefix: int,
                 prompt: np.ndarray, max_steps: int, stop_on_eos: bool = True,
                 with_logits: bool = False):
    """kcache/vcache: [L, cap, D] uint16 (modified in place).  Returns (tokens, margins)
    or (tokens, margins, last_logits)."""
    d, w = t2s_structs(model)
    cap = kcache.shape[1]
    pr = np.ascontiguousarray(prompt, np.int32)
    toks = np.zeros(max_steps, dtype=np.int32)
    margins = np.zeros(max_steps, dtype=np.float32)
    logits = np.zeros(model["vocab"], dtype=np.float32)
    n = lib().ora_t2s_generate(ctypes.byref(d), ctypes.byref(w), _p(kcache), _p(vcache), cap,
                               prefix, _p(pr), pr.size, max_steps, int(stop_on_eos), _p(toks),
                               _p(margins), _p(logits))
    if n < 0:
        raise ValueError("ora_t2s_generate: cache too small")
    if with_logits:
        return toks[:n], margins, logits
    return toks[:n], margins


def t2s_generate_ex(model: dict, kcache: np.ndarray, vcache: np.ndarray, prefix: int,
                    prompt: np.ndarray, max_steps: int, stop_on_eos: bool = False,
                    literal: bool = False):
    """ora_t2s_generate_ex: (tokens, margins, logits [steps, vocab]).  literal
    selects the line-by-line restatement of the reference's decode layer."""
    d, w = t2s_structs(model)
    cap = kcache.shape[1]
    pr = np.ascontiguousarray(prompt, np.int32)
    toks = np.zeros(max_steps, dtype=np.int32)
    margins = np.zeros(max_steps, dtype=np.float32)
    logits = np.zeros((max_steps, model["vocab"]), dtype=np.float32)
    n = lib().ora_t2s_generate_ex(ctypes.byref(d), ctypes.byref(w), _p(kcache), _p(vcache), cap,
                                  prefix, _p(pr), pr.size, max_steps, int(stop_on_eos),
                                  int(literal), _p(toks), _p(margins), _p(logits))
    if n < 0:
        raise ValueError("ora_t2s_generate_ex: cache too small")
    return toks[:n], margins, logits


class Sampling(ctypes.Structure):
    """SamplingParams (t2s_engine.hpp:69-77); mode 0 greedy, 1 top-k."""
    _fields_ = [("mode", c_int), ("top_k", c_int), ("top_p", ctypes.c_float),
                ("temperature", ctypes.c_float), ("rep_penalty", ctypes.c_float),
                ("seed", ctypes.c_ulonglong)]


def t2s_generate_sampled(model: dict, kcache: np.ndarray, vcache: np.ndarray, prefix: int,
                         prompt: np.ndarray, max_steps: int, sampling: "Sampling",
                         stop_on_eos: bool = True):
    """(tokens, margins) of a generate that samples with `sampling`."""
    d, w = t2s_structs(model)
    cap = kcache.shape[1]
    pr = np.ascontiguousarray(prompt, np.int32)
    toks = np.zeros(max_steps, dtype=np.int32)
    margins = np.zeros(max_steps, dtype=np.float32)
    n = lib().ora_t2s_generate_sampled(ctypes.byref(d), ctypes.byref(w), _p(kcache), _p(vcache),
                                       cap, prefix, _p(pr), pr.size, max_steps, int(stop_on_eos),
                                       ctypes.byref(sampling), _p(toks), _p(margins))
    if n < 0:
        raise ValueError("ora_t2s_generate_sampled: cache too small")
    return toks[:n], margins


def t2s_decode_layer_literal(model: dict, layer: int, x: np.ndarray, pos: int, kc: np.ndarray,
                             vc: np.ndarray) -> None:
    d, w = t2s_structs(model)
    lib().ora_t2s_decode_layer_literal(ctypes.byref(d), ctypes.byref(w), layer, _p(x), pos,
                                       _p(kc), _p(vc))


def encoder_layer(model: dict, layer: int, x: np.ndarray, B: int, T: int, valid=None) -> None:
    """x [B*T, C] fp32, updated in place (model: workloads.encoder_model)."""
    d = EncoderDims(model["layers"], model["hidden"], model["heads"], model["ffn"], model["eps"])
    w = EncoderWeights(*[_p(model[n]) for n in ("wqkv", "bqkv", "wo", "bo", "ln1g", "ln1b", "wi",
                                                "bi", "wf", "bf", "ln2g", "ln2b")])
    vd = None if valid is None else np.ascontiguousarray(valid, np.int32)
    lib().ora_encoder_layer(ctypes.byref(d), ctypes.byref(w), layer, _p(x), B, T, _p(vd))


class HubertFrontCfg(ctypes.Structure):
    _fields_ = [("conv_dim", c_int * 7), ("conv_kernel", c_int * 7), ("conv_stride", c_int * 7),
                ("hidden", c_int), ("pos_k", c_int), ("pos_groups", c_int),
                ("ln_eps", ctypes.c_double)]


class HubertFrontWeights(ctypes.Structure):
    _fields_ = [("conv_w", c_void_p * 7)] + [(n, c_void_p) for n in (
        "gn_g", "gn_b", "proj_ln_g", "proj_ln_b", "proj_w", "proj_b", "pos_w", "pos_b",
        "enc_ln_g", "enc_ln_b")]


def hubert_front(model: dict, wav: np.ndarray) -> np.ndarray:
    """hubert.cpp:476-580 on the CPU: waveform -> [frames][hidden]."""
    c = HubertFrontCfg((c_int * 7)(*model["conv_dim"]), (c_int * 7)(*model["conv_kernel"]),
                       (c_int * 7)(*model["conv_stride"]), model["hidden"], model["pos_k"],
                       model["pos_groups"], model["ln_eps"])
    w = HubertFrontWeights((c_void_p * 7)(*[_p(a) for a in model["conv_w"]]),
                           *[_p(model[n]) for n in ("gn_g", "gn_b", "proj_ln_g", "proj_ln_b",
                                                    "proj_w", "proj_b", "pos_w", "pos_b",
                                                    "enc_ln_g", "enc_ln_b")])
    wav = np.ascontiguousarray(wav, np.float32)
    T = lib().ora_hubert_front_frames(ctypes.byref(c), wav.size)
    out = np.zeros((T, model["hidden"]), np.float32)
    lib().ora_hubert_front(ctypes.byref(c), ctypes.byref(w), _p(wav), wav.size, _p(out))
    return out


class Named(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("f32", c_void_p), ("f16", c_void_p),
                ("numel", ctypes.c_uint64)]


class SovitsLatentCfg(ctypes.Structure):
    _fields_ = [(n, c_int) for n in (
        "ssl_dim", "hidden", "filter", "heads", "kernel", "window", "layers_ssl", "layers_text",
        "layers_2", "mrte_hidden", "mrte_heads", "gin", "flows", "wn_layers", "wn_kernel")] + [
        ("noise_scale", c_float)]


def named_tensors(tensors: dict):
    """(ctypes array, keep-alive list) of ora_named for a name -> array dict:
    uint16 arrays are fp16 bits, float32 arrays fp32."""
    keep, arr = [], (Named * len(tensors))()
    for i, (k, a) in enumerate(tensors.items()):
        a = np.ascontiguousarray(a)
        keep.append(a)
        f16 = a.dtype == np.uint16
        arr[i] = Named(k.encode(), None if f16 else a.ctypes.data, a.ctypes.data if f16 else None,
                       a.size)
    return arr, keep


def sovits_latent(model: dict, codes, phones, ge, ge_text, noise=None):
    """sovits_engine.hpp:48-93 steps 1-5 on the CPU: (m_p, logs_p, z), each
    [hidden][2 * len(codes)]; raises ValueError on the oracle's error codes."""
    c = SovitsLatentCfg(*[model[f[0]] for f in SovitsLatentCfg._fields_])
    arr, keep = named_tensors(model["tensors"])
    codes = np.ascontiguousarray(codes, np.int64)
    phones = np.ascontiguousarray(phones, np.int64)
    ge = np.ascontiguousarray(ge, np.float32)
    ge_text = np.ascontiguousarray(ge_text, np.float32)
    Tq = 2 * codes.size
    outs = [np.zeros((model["hidden"], Tq), np.float32) for _ in range(3)]
    nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
    rc = lib().ora_sovits_latent(ctypes.byref(c), arr, len(keep), _p(codes), codes.size,
                                 _p(phones), phones.size, _p(ge), _p(ge_text), _p(nz),
                                 *[_p(o) for o in outs])
    if rc:
        raise ValueError(f"ora_sovits_latent: {rc}")
    return tuple(outs)


def sv_forward(model: dict, fbank: np.ndarray) -> np.ndarray:
    """sv.cpp forward3 on the CPU: fbank [frames][n_mels] -> embedding."""
    arr, keep = named_tensors(model["tensors"])
    fb = np.ascontiguousarray(fbank, np.float32)
    frames, n_mels = fb.shape
    emb = np.zeros(model["emb_channels"] * (n_mels // 8 + 1), np.float32)
    n = lib().ora_sv_forward(arr, len(keep), _p(fb), frames, n_mels, _p(emb))
    if n == 0:
        raise ValueError("ora_sv_forward: missing tensor")
    return emb[:n].copy()


def sv_conv2d_f16(x: np.ndarray, w16: np.ndarray, stride: int, pad: int) -> np.ndarray:
    """conv2d_f16: x [c_in][h][w] fp32, w16 [c_out][c_in][kh][kw] fp16 bits."""
    x = np.ascontiguousarray(x, np.float32)
    w16 = np.ascontiguousarray(w16, np.uint16)
    c_in, h, w = x.shape
    c_out, _, kh, kw = w16.shape
    oh, ow = (h + 2 * pad - kh) // stride + 1, (w + 2 * pad - kw) // stride + 1
    out = np.zeros((c_out, oh, ow), np.float32)
    lib().ora_sv_conv2d_f16(_p(x), c_in, h, w, _p(w16), c_out, kh, kw, stride, pad, _p(out))
    return out
