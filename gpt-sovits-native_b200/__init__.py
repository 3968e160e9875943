"""gsv_b200 — Python view of libgsvk.so, the B200 build of the GPT-SoVITS-native
`src/kern` GEMM/GEMV hot path.

Everything here is a thin ctypes layer over the C ABI declared in
include/gsvk.h; all arithmetic happens in the CUDA kernels of libgsvk.so.
There is no CPU fallback: if libgsvk.so is missing or no sm_100 device is
present, calls raise.

Tensors are torch CUDA tensors (torch is used for device memory and streams
only).  fp16 bit patterns travel as torch.float16 tensors.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_char, c_double, c_float, c_int, c_size_t, c_void_p

from . import replicas  # noqa: F401  (multi-GPU host logic: shards, barriers, gathers)
from . import workloads  # noqa: F401  (seeded synthetic inputs)

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgsvk.so")

ACT_NONE, ACT_RELU, ACT_GELU_ERF, ACT_LEAKY, ACT_TANH = 0, 1, 2, 3, 4
STATUS = {0: "OK", -1: "INVALID", -2: "ALIGN", -3: "CUDA", -4: "TIMEOUT", -5: "UNSUPPORTED",
          -6: "NOMEM", -7: "NODEV"}


class GsvkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"gsvk error {code} ({STATUS.get(code, '?')}): {msg}")
        self.code = code


_lib = None

# name -> (restype, argtypes); the exported surface of include/gsvk.h.
_vp, _sz = c_void_p, c_size_t
SIGNATURES = {
    "gsvk_version": (c_int, []),
    "gsvk_last_error": (ctypes.c_char_p, []),
    "gsvk_device_init": (c_int, [c_int]),
    "gsvk_available": (c_int, []),
    "gsvk_device_status": (c_int, [c_int]),
    "gsvk_gemm_f16": (c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "gsvk_gemm_f16_ex": (c_int, [_vp, _vp]),
    "gsvk_gemm_grouped_f16": (c_int, [_vp, _sz, _vp]),
    "gsvk_gemm_f16_batched": (c_int, [_vp, _sz, _sz, _sz, _sz, _vp]),
    "gsvk_gemm_set_pair": (c_int, [c_int]),
    "gsvk_gemm_uses_pair": (c_int, [c_size_t, c_size_t, c_size_t]),
    "gsvk_gemm_set_bulk_epilogue": (c_int, [c_int]),
    "gsvk_weights_register": (c_int, [_vp, _sz, _sz, _vp]),
    "gsvk_weights_release": (c_int, [_vp]),
    "gsvk_weights_data": (_vp, [_vp]),
    "gsvk_gemm_f16_w": (c_int, [_vp, _vp, _vp]),
    "gsvk_gemv_f16w_f32acc_w": (c_int, [_vp, _vp, _vp, _vp]),
    "gsvk_f32_to_f16": (c_int, [_vp, _vp, _sz, _vp]),
    "gsvk_f16_to_f32": (c_int, [_vp, _vp, _sz, _vp]),
    "gsvk_gemv_f16w_f32acc": (c_int, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "gsvk_gemv_f16x_fmlal": (c_int, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "gsvk_gemv_ex": (c_int, [_vp, _vp, c_int, _vp, _vp, _sz, _sz, _vp, _vp, c_int, c_float, _vp]),
    "gsvk_t2s_create": (c_int, [_vp, _vp, _vp]),
    "gsvk_t2s_destroy": (c_int, [_vp]),
    "gsvk_t2s_load_kv": (c_int, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "gsvk_t2s_prefill": (c_int, [_vp, _vp, _sz, _sz, _sz, _vp]),
    "gsvk_t2s_generate": (c_int, [_vp, _sz, _vp, _sz, _sz, c_int, _vp, _vp, _vp, _vp]),
    "gsvk_t2s_generate_device": (c_int, [_vp, _sz, _vp, _sz, _sz, c_int, _vp, _vp, _vp, _vp]),
    "gsvk_t2s_read_logits": (c_int, [_vp, _vp]),
    "gsvk_t2s_prompt": (c_int, [_vp, _sz, _vp, _sz, _vp]),
    "gsvk_t2s_decode": (c_int, [_vp, _sz, _vp, _sz, _sz, c_int, _vp, _vp, _vp, _vp]),
    "gsvk_t2s_launches_per_generate": (c_int, [_vp]),
    "gsvk_t2s_set_trace": (c_int, [_vp, c_int]),
    "gsvk_t2s_set_decode_kernel": (c_int, [_vp, c_int]),
    "gsvk_t2s_read_kv": (c_int, [_vp, _vp, _vp]),
    "gsvk_t2s_set_decode_ctas": (c_int, [_vp, c_int]),
    "gsvk_t2s_decode_kernel": (c_int, [_vp]),
    "gsvk_t2s_set_sampling": (c_int, [_vp, _vp]),
    "gsvk_set_spin_limit_for_test": (c_int, [ctypes.c_uint32]),
    "gsvk_test_rstd": (c_int, [_vp, _vp, _sz, _vp]),
    "gsvk_hubert_front_create": (c_int, [_vp, _vp, _vp]),
    "gsvk_hubert_front_destroy": (c_int, [_vp]),
    "gsvk_hubert_front_frames": (_sz, [_vp, _sz]),
    "gsvk_hubert_front_forward": (c_int, [_vp, _vp, _sz, _vp, _vp]),
    "gsvk_gsv_open": (c_int, [ctypes.c_char_p, _vp]),
    "gsvk_gsv_close": (c_int, [_vp]),
    "gsvk_gsv_count": (_sz, [_vp]),
    "gsvk_gsv_model_name": (ctypes.c_char_p, [_vp]),
    "gsvk_gsv_config": (ctypes.c_char_p, [_vp, _vp]),
    "gsvk_gsv_tensor_at": (c_int, [_vp, _sz, _vp]),
    "gsvk_gsv_find": (c_int, [_vp, ctypes.c_char_p, _vp]),
    "gsvk_t2s_create_from_gsv": (c_int, [_vp, c_int, _vp]),
    "gsvk_sv_create": (c_int, [_vp, _vp, _sz, _vp]),
    "gsvk_sv_create_from_gsv": (c_int, [_vp, _vp, _vp]),
    "gsvk_sv_destroy": (c_int, [_vp]),
    "gsvk_sv_embedding_size": (_sz, [_vp]),
    "gsvk_sv_forward": (c_int, [_vp, _vp, _sz, _vp, _vp]),
    "gsvk_sovits_latent_create": (c_int, [_vp, _vp, _sz, _vp]),
    "gsvk_sovits_latent_create_from_gsv": (c_int, [_vp, _vp, _vp]),
    "gsvk_sovits_latent_destroy": (c_int, [_vp]),
    "gsvk_sovits_latent_forward": (c_int, [_vp, _vp, _sz, _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp,
                                           _vp]),
    "gsvk_t2s_read_trace": (c_int, [_vp, _vp, _sz]),
    "gsvk_attention_workspace_floats": (_sz, [_sz, _sz, _sz]),
    "gsvk_attention_decode": (c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, c_float, _vp, _vp, _vp]),
    "gsvk_attention_decode_noalloc_max_floats": (_sz, []),
    "gsvk_attention_decode_noalloc": (c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, c_float, _vp,
                                              _vp]),
    "gsvk_conv1d_pack_weight": (c_int, [_vp, _sz, _sz, _sz, _vp, _vp]),
    "gsvk_convt1d_pack_weight": (c_int, [_vp, _sz, _sz, _sz, _vp, _vp]),
    "gsvk_conv1d_f16": (c_int, [_vp, _vp]),
    "gsvk_convt1d_f16": (c_int, [_vp, _vp]),
    "gsvk_channels_to_rows_f16": (c_int, [_vp, _sz, _sz, _vp, _vp]),
    "gsvk_rows_to_channels_f32": (c_int, [_vp, _sz, _sz, _vp, _vp]),
    "gsvk_decoder_out_len": (_sz, [_vp, _sz]),
    "gsvk_decoder_create": (c_int, [_vp, _vp, _vp, _vp]),
    "gsvk_decoder_destroy": (c_int, [_vp]),
    "gsvk_decoder_forward": (c_int, [_vp, _vp, _sz, _vp, _vp]),
    "gsvk_decoder_launches": (c_int, [_vp]),
    "gsvk_decoder_set_graph": (c_int, [_vp, c_int]),
    "gsvk_sgemm": (c_int, [c_char, c_char, c_int, c_int, c_int, c_float, _vp, c_int, _vp, c_int,
                           c_float, _vp, c_int, _vp]),
    "gsvk_gemm_nt_f16w": (c_int, [_vp, _sz, _sz, _vp, _sz, _vp, _vp]),
    "gsvk_device_alloc_copy": (c_int, [_vp, _sz, _vp]),
    "gsvk_device_free": (c_int, [_vp]),
    "gsvk_gemm_chain_run": (c_int, [_vp, _sz, _vp]),
    "gsvk_encoder_create": (c_int, [_vp, _vp, _vp]),
    "gsvk_encoder_destroy": (c_int, [_vp]),
    "gsvk_encoder_forward": (c_int, [_vp, _vp, _sz, _sz, _vp, _vp]),
    "gsvk_encoder_launches": (c_int, [_vp]),
    "gsvk_t2s_batch_create": (c_int, [_vp, _vp, c_int, c_int, _vp]),
    "gsvk_t2s_batch_destroy": (c_int, [_vp]),
    "gsvk_t2s_batch_load_kv": (c_int, [_vp, c_int, _vp, _vp, _sz, _sz, _vp]),
    "gsvk_t2s_batch_begin": (c_int, [_vp, c_int, _vp, _vp, _vp, _vp, c_int, _vp]),
    "gsvk_t2s_batch_run": (c_int, [_vp, c_int, c_int, _vp]),
    "gsvk_t2s_batch_read": (c_int, [_vp, c_int, _vp, _vp]),
    "gsvk_t2s_batch_read_logits": (c_int, [_vp, _vp]),
    "gsvk_t2s_batch_launches_per_step": (c_int, [_vp]),
    "gsvk_t2s_batch_set_attention": (c_int, [c_void_p, c_int]),
    "gsvk_t2s_batch_attention": (c_int, [c_void_p]),
    "gsvk_layernorm_rows": (c_int, [_vp, _vp, _vp, _vp, _sz, _sz, c_double, _vp]),
    "gsvk_softmax_rows": (c_int, [_vp, _vp, _sz, _sz, _vp]),
    "gsvk_activation": (c_int, [_vp, _vp, _sz, c_int, c_float, _vp]),
}


def lib():
    """Load libgsvk.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} not built: run `make -C {_HERE}` "
                              "(or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().gsvk_last_error().decode(errors="replace")


def check(rc: int) -> None:
    if rc != 0:
        raise GsvkError(rc, last_error())


def device_init(device: int = 0) -> None:
    check(lib().gsvk_device_init(device))


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("gsvk takes CUDA tensors")
    if t.dim() > 0 and t.stride(-1) != 1:
        raise ValueError("gsvk takes tensors with unit inner stride")
    return t.data_ptr()


def _stream(stream):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


# ---------------------------------------------------------------------- a4
def f32_to_f16(src, dst=None, stream=None):
    import torch

    dst = dst if dst is not None else torch.empty(src.shape, dtype=torch.float16, device=src.device)
    check(lib().gsvk_f32_to_f16(_ptr(src), _ptr(dst), src.numel(), _stream(stream)))
    return dst


def f16_to_f32(src, dst=None, stream=None):
    import torch

    dst = dst if dst is not None else torch.empty(src.shape, dtype=torch.float32, device=src.device)
    check(lib().gsvk_f16_to_f32(_ptr(src), _ptr(dst), src.numel(), _stream(stream)))
    return dst


# ------------------------------------------------------------------ a1, a2
def gemv_f16w_f32acc(w, x, y=None, stream=None):
    """kern::gemv_f16w_f32acc: y[out] = W[out,in] (fp16) . x[in] (fp32)."""
    import torch

    out_, in_ = w.shape
    y = y if y is not None else torch.empty(out_, dtype=torch.float32, device=w.device)
    check(lib().gsvk_gemv_f16w_f32acc(_ptr(w), _ptr(x), _ptr(y), out_, in_, _stream(stream)))
    return y


def gemv_f16x_fmlal(w, xh, y=None, stream=None):
    """kern::gemv_f16x_fmlal: fp16 x, fp32 accumulate."""
    import torch

    out_, in_ = w.shape
    y = y if y is not None else torch.empty(out_, dtype=torch.float32, device=w.device)
    check(lib().gsvk_gemv_f16x_fmlal(_ptr(w), _ptr(xh), _ptr(y), out_, in_, _stream(stream)))
    return y


def gemv_ex(w, x, bias=None, residual=None, act=ACT_NONE, slope=0.0, y=None, y_f16=None,
            stream=None):
    import torch

    out_, in_ = w.shape
    if y is None:
        y = torch.empty(out_, dtype=torch.float32, device=w.device)
    check(lib().gsvk_gemv_ex(_ptr(w), _ptr(x), int(x.dtype == torch.float16), _ptr(y), _ptr(y_f16),
                             out_, in_, _ptr(bias), _ptr(residual), act, slope, _stream(stream)))
    return y


# ------------------------------------------------------------- a3, a6, a9
class GemmArgs(ctypes.Structure):
    _fields_ = [("a", _vp), ("lda", _sz), ("b", _vp), ("ldb", _sz), ("M", _sz), ("N", _sz),
                ("K", _sz), ("bias", _vp), ("residual", _vp), ("ld_res", _sz), ("c", _vp),
                ("ldc", _sz), ("c_f16", _vp), ("ldc_f16", _sz), ("act", c_int), ("slope", c_float),
                ("alpha", c_float)]


def _gemm_args(a, b, bias=None, residual=None, act=ACT_NONE, slope=0.0, alpha=1.0, c=None,
               c_f16=None):
    M, K = a.shape
    N = b.shape[0]
    return GemmArgs(_ptr(a), a.stride(0), _ptr(b), b.stride(0), M, N, K, _ptr(bias), _ptr(residual),
                    0 if residual is None else residual.stride(0), _ptr(c),
                    0 if c is None else c.stride(0), _ptr(c_f16),
                    0 if c_f16 is None else c_f16.stride(0), act, slope, alpha)


PAIR_NEVER, PAIR_AUTO, PAIR_ALWAYS = 0, 1, 2


def gemm_set_pair(mode):
    """Two-SM (cta_group::2) GEMM kernel for eligible plain problems: PAIR_AUTO
    (the default, when its tile rounds cost no more), PAIR_ALWAYS or
    PAIR_NEVER; True / False mean PAIR_AUTO / PAIR_NEVER."""
    if mode is True or mode is False:
        mode = PAIR_AUTO if mode else PAIR_NEVER
    check(lib().gsvk_gemm_set_pair(int(mode)))


def gemm_set_bulk_epilogue(enable: bool):
    """One-SM kernel: bulk-copy epilogue where possible (default) or per-row
    stores everywhere (identical results)."""
    check(lib().gsvk_gemm_set_bulk_epilogue(int(bool(enable))))


def gemm_uses_pair(M: int, N: int, K: int) -> bool:
    """Whether an M x N x K gemm_ex call runs on the two-SM kernel."""
    return bool(lib().gsvk_gemm_uses_pair(int(M), int(N), int(K)))


def gemm_batched(a, b, bias=None, residual=None, act=ACT_NONE, slope=0.0, alpha=1.0, c=None,
                 c_f16=None, stream=None):
    """Strided batched C[i] = act(alpha * A[i].B[i]^T + bias) + residual[i]:
    a [batch, M, K], b [batch, N, K] or [N, K] (shared), outputs and
    residual [batch, M, N] (CUDA tensors, rows contiguous)."""
    batch, M, K = a.shape
    N = b.shape[-2]
    out = c if c is not None else c_f16
    g = GemmArgs(_ptr(a), a.stride(1), _ptr(b), b.stride(-2), M, N, K, _ptr(bias),
                 _ptr(residual), 0 if residual is None else residual.stride(1), _ptr(c),
                 0 if c is None else c.stride(1), _ptr(c_f16),
                 0 if c_f16 is None else c_f16.stride(1), act, slope, alpha)
    sb = b.stride(0) if b.dim() == 3 else 0
    check(lib().gsvk_gemm_f16_batched(ctypes.byref(g), batch, a.stride(0), sb, out.stride(0),
                                      _stream(stream)))
    return out


def gemm_grouped(problems, stream=None):
    """Independent GEMMs submitted together: `problems` is a list of dicts of
    gemm_ex keyword arguments (a, b, bias, residual, act, slope, alpha, c, c_f16)."""
    arr = (GemmArgs * len(problems))(*[_gemm_args(**p) for p in problems])
    check(lib().gsvk_gemm_grouped_f16(arr, len(problems), _stream(stream)))


class GemmChainLink(ctypes.Structure):
    _fields_ = [("chain_id", c_int), ("depth", c_int), ("gemm", GemmArgs)]


def gemm_chain_run(links, stream=None):
    """AmxChainLink / amx_chain_run: `links` is a list of (chain_id, depth,
    dict of gemm_ex keyword arguments); links of one chain run in depth
    order, chains are independent."""
    arr = (GemmChainLink * len(links))(*[GemmChainLink(c, d, _gemm_args(**g)) for c, d, g in links])
    check(lib().gsvk_gemm_chain_run(arr, len(links), _stream(stream)))


def gemm_nt_f16w(x, w, y=None, stream=None):
    """accel::gemm_nt_f16w: y[T, out] = x[T, in] (fp32) . W[out, in]^T (fp16,
    widened exactly), fp32 accumulation."""
    import torch

    T, in_ = x.shape
    out_ = w.shape[0]
    y = y if y is not None else torch.empty(T, out_, dtype=torch.float32, device=x.device)
    check(lib().gsvk_gemm_nt_f16w(_ptr(x), T, in_, _ptr(w), out_, _ptr(y), _stream(stream)))
    return y


class Weights:
    """A registered [rows, cols] fp16 weight (host numpy uint16 or a CUDA tensor)."""

    def __init__(self, w, rows: int = None, cols: int = None):
        if hasattr(w, "ctypes"):
            rows, cols = w.shape
            ptr = w.ctypes.data
        else:
            rows, cols = w.shape
            ptr = w.data_ptr()
        self.rows, self.cols = int(rows), int(cols)
        h = ctypes.c_void_p()
        check(lib().gsvk_weights_register(ptr, self.rows, self.cols, ctypes.byref(h)))
        self.h = h

    def data_ptr(self) -> int:
        return lib().gsvk_weights_data(self.h)

    def gemm(self, a, bias=None, residual=None, act=ACT_NONE, slope=0.0, alpha=1.0, c=None,
             c_f16=None, stream=None):
        M, K = a.shape
        g = GemmArgs(_ptr(a), a.stride(0), None, 0, M, self.rows, K, _ptr(bias), _ptr(residual),
                     0 if residual is None else residual.stride(0), _ptr(c),
                     0 if c is None else c.stride(0), _ptr(c_f16),
                     0 if c_f16 is None else c_f16.stride(0), act, slope, alpha)
        check(lib().gsvk_gemm_f16_w(ctypes.byref(g), self.h, _stream(stream)))
        return c if c is not None else c_f16

    def gemv(self, x, y, stream=None):
        check(lib().gsvk_gemv_f16w_f32acc_w(self.h, _ptr(x), _ptr(y), _stream(stream)))
        return y

    def close(self):
        if getattr(self, "h", None):
            lib().gsvk_weights_release(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_status(reset: bool = True) -> int:
    """0, or GSVK_ERR_TIMEOUT (-4) if a bounded device wait gave up."""
    return lib().gsvk_device_status(int(reset))


def gemm_f16(a, b, c=None, stream=None):
    """kern::gemm_f16x_fmlal: C[M,N] = A[M,K] . B[N,K]^T (fp16 in, fp32 out)."""
    import torch

    M, K = a.shape
    N = b.shape[0]
    c = c if c is not None else torch.empty(M, N, dtype=torch.float32, device=a.device)
    check(lib().gsvk_gemm_f16(_ptr(a), _ptr(b), _ptr(c), M, N, K, _stream(stream)))
    return c


def gemm_ex(a, b, bias=None, residual=None, act=ACT_NONE, slope=0.0, alpha=1.0, c=None,
            c_f16=None, stream=None):
    """C = act(alpha * A.B^T + bias) + residual -> fp32 c and/or fp16 c_f16."""
    M, K = a.shape
    N = b.shape[0]
    g = GemmArgs(_ptr(a), a.stride(0), _ptr(b), b.stride(0), M, N, K, _ptr(bias), _ptr(residual),
                 0 if residual is None else residual.stride(0), _ptr(c),
                 0 if c is None else c.stride(0), _ptr(c_f16),
                 0 if c_f16 is None else c_f16.stride(0), act, slope, alpha)
    check(lib().gsvk_gemm_f16_ex(ctypes.byref(g), _stream(stream)))
    return c if c is not None else c_f16


# ------------------------------------------------------- decode attention
def attention_workspace_floats(length: int, n_heads: int, head_dim: int) -> int:
    return lib().gsvk_attention_workspace_floats(length, n_heads, head_dim)


def attention_decode(q, kcache, vcache, length: int, n_heads: int, head_dim: int, scale: float,
                     out=None, workspace=None, stream=None):
    """One decode step of multi-head attention over a token-major fp16 cache."""
    import torch

    out = out if out is not None else torch.empty(n_heads * head_dim, device=q.device)
    if workspace is None:
        workspace = torch.empty(attention_workspace_floats(length, n_heads, head_dim),
                                device=q.device)
    check(lib().gsvk_attention_decode(_ptr(q), _ptr(kcache), _ptr(vcache), length, n_heads,
                                      head_dim, kcache.stride(0), scale, _ptr(out),
                                      _ptr(workspace), _stream(stream)))
    return out


# ---------------------------------------------------------------------- a5
def sgemm(ta: str, tb: str, M: int, N: int, K: int, alpha: float, A, lda: int, B, ldb: int,
          beta: float, C, ldc: int, stream=None):
    """accel::sgemm on device fp32 buffers (row-major, cblas semantics)."""
    check(lib().gsvk_sgemm(ta.encode(), tb.encode(), M, N, K, alpha, _ptr(A), lda, _ptr(B), ldb,
                           beta, _ptr(C), ldc, _stream(stream)))
    return C


# --------------------------------------------------------------------- a22
def layernorm_rows(x, g, b, eps, y=None, stream=None):
    import torch

    n = x.shape[-1]
    y = y if y is not None else torch.empty_like(x)
    check(lib().gsvk_layernorm_rows(_ptr(x), _ptr(g), _ptr(b), _ptr(y), x.numel() // n, n, eps,
                                    _stream(stream)))
    return y


def softmax_rows(x, y=None, stream=None):
    import torch

    n = x.shape[-1]
    y = y if y is not None else torch.empty_like(x)
    check(lib().gsvk_softmax_rows(_ptr(x), _ptr(y), x.numel() // n, n, _stream(stream)))
    return y


def activation(x, act, slope=0.0, y=None, stream=None):
    import torch

    y = y if y is not None else torch.empty_like(x)
    check(lib().gsvk_activation(_ptr(x), _ptr(y), x.numel(), act, slope, _stream(stream)))
    return y


# ------------------------------------------------------------ a16 - a19: T2S
class T2SConfig(ctypes.Structure):
    _fields_ = [("n_layers", c_int), ("d_model", c_int), ("n_heads", c_int), ("ffn", c_int),
                ("vocab", c_int), ("ln_eps", c_float), ("alpha_audio", c_float), ("cap", c_int)]


class T2SHostWeights(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("wqkv", "bqkv", "wout", "bout", "w1", "b1", "w2", "b2",
                                   "n1g", "n1b", "n2g", "n2b", "wpred", "audio_emb")]


class HubertFrontConfig(ctypes.Structure):
    _fields_ = [("conv_dim", c_int * 7), ("conv_kernel", c_int * 7), ("conv_stride", c_int * 7),
                ("hidden", c_int), ("pos_k", c_int), ("pos_groups", c_int), ("ln_eps", c_float),
                ("max_samples", _sz)]


class HubertFrontWeights(ctypes.Structure):
    _fields_ = [("conv_w", _vp * 7)] + [(n, _vp) for n in (
        "gn_g", "gn_b", "proj_ln_g", "proj_ln_b", "proj_w", "proj_b", "pos_w", "pos_b",
        "enc_ln_g", "enc_ln_b")]


class HubertFront:
    """HuBERT feature front-end (gsvk_hubert_front_*): waveform -> encoder input."""

    NAMES = ("gn_g", "gn_b", "proj_ln_g", "proj_ln_b", "proj_w", "proj_b", "pos_w", "pos_b",
             "enc_ln_g", "enc_ln_b")

    def __init__(self, model: dict, max_samples: int):
        import numpy as np

        self.hidden = model["hidden"]
        conv = [np.ascontiguousarray(w) for w in model["conv_w"]]
        keep = {n: np.ascontiguousarray(model[n]) for n in self.NAMES}
        cfg = HubertFrontConfig((c_int * 7)(*model["conv_dim"]), (c_int * 7)(*model["conv_kernel"]),
                                (c_int * 7)(*model["conv_stride"]), model["hidden"],
                                model["pos_k"], model["pos_groups"], model["ln_eps"], max_samples)
        w = HubertFrontWeights((_vp * 7)(*[a.ctypes.data for a in conv]),
                               *[keep[n].ctypes.data for n in self.NAMES])
        h = c_void_p()
        check(lib().gsvk_hubert_front_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(h)))
        self.h = h

    def frames(self, n: int) -> int:
        return lib().gsvk_hubert_front_frames(self.h, n)

    def forward(self, wav, x=None, stream=None):
        import torch

        n = wav.numel()
        x = x if x is not None else torch.empty(self.frames(n), self.hidden, device=wav.device)
        check(lib().gsvk_hubert_front_forward(self.h, _ptr(wav), n, _ptr(x), _stream(stream)))
        return x

    def close(self):
        if self.h:
            lib().gsvk_hubert_front_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GsvTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("rank", ctypes.c_uint32),
                ("dims", ctypes.c_uint32 * 8), ("src_dtype", c_int), ("numel", ctypes.c_uint64),
                ("f32", _vp), ("f16", _vp)]


def gsv_tensors(tensors: dict):
    """(ctypes array of GsvTensor, keep-alive list) for a name -> array dict:
    uint16 arrays are fp16 bits, float32 arrays fp32 (the .gsv tensor view)."""
    import numpy as np

    keep, arr = [], (GsvTensor * len(tensors))()
    for i, (k, a) in enumerate(tensors.items()):
        a = np.ascontiguousarray(a)
        name = k.encode()
        keep += [a, name]
        f16 = a.dtype == np.uint16
        dims = (ctypes.c_uint32 * 8)(*a.shape)
        arr[i] = GsvTensor(name, a.ndim, dims, 2 if f16 else 1, a.size,
                           None if f16 else a.ctypes.data, a.ctypes.data if f16 else None)
    return arr, keep


class SovitsLatentConfig(ctypes.Structure):
    _fields_ = [(n, c_int) for n in (
        "ssl_dim", "hidden", "filter", "heads", "kernel", "window", "layers_ssl", "layers_text",
        "layers_2", "mrte_hidden", "mrte_heads", "gin", "flows", "wn_layers", "wn_kernel")] + [
        ("noise_scale", c_float), ("max_codes", _sz), ("max_phones", _sz)]


class SovitsLatent:
    """SoVITS latent path (gsvk_sovits_latent_*): codes + phones + speaker
    embeddings -> z [hidden][2 n_codes], the generator's input."""

    def __init__(self, model: dict, max_codes: int, max_phones: int, gsv: "GsvFile" = None):
        self.hidden = model["hidden"]
        names = [f[0] for f in SovitsLatentConfig._fields_[:-2]]
        self.cfg = SovitsLatentConfig(*[model[n] for n in names], max_codes, max_phones)
        h = c_void_p()
        if gsv is not None:
            check(lib().gsvk_sovits_latent_create_from_gsv(gsv.h, ctypes.byref(self.cfg),
                                                          ctypes.byref(h)))
        else:
            arr, keep = gsv_tensors(model["tensors"])
            check(lib().gsvk_sovits_latent_create(ctypes.byref(self.cfg), arr, len(arr),
                                                  ctypes.byref(h)))
        self.h = h

    def forward(self, codes, phones, ge, ge_text, noise=None, z=None, m_p=None, logs_p=None,
                stream=None):
        """codes, phones: host int64 arrays; ge, ge_text, noise: device fp32."""
        import numpy as np
        import torch

        codes = np.ascontiguousarray(codes, np.int64)
        phones = np.ascontiguousarray(phones, np.int64)
        Tq = 2 * codes.size
        if z is None:
            z = torch.empty(self.hidden, Tq, device=ge.device)
        check(lib().gsvk_sovits_latent_forward(self.h, codes.ctypes.data, codes.size,
                                               phones.ctypes.data, phones.size, _ptr(ge),
                                               _ptr(ge_text), _ptr(noise), _ptr(z), _ptr(m_p),
                                               _ptr(logs_p), _stream(stream)))
        return z

    def close(self):
        if self.h:
            lib().gsvk_sovits_latent_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SvConfig(ctypes.Structure):
    _fields_ = [("n_mels", c_int), ("max_frames", _sz)]


class SvEncoder:
    """SV speaker encoder (gsvk_sv_*): fbank [frames][n_mels] -> embedding."""

    def __init__(self, model: dict, max_frames: int, n_mels: int = 80, gsv: "GsvFile" = None):
        self.cfg = SvConfig(n_mels, max_frames)
        h = c_void_p()
        if gsv is not None:
            check(lib().gsvk_sv_create_from_gsv(gsv.h, ctypes.byref(self.cfg), ctypes.byref(h)))
        else:
            arr, keep = gsv_tensors(model["tensors"])
            check(lib().gsvk_sv_create(ctypes.byref(self.cfg), arr, len(arr), ctypes.byref(h)))
        self.h = h

    def embedding_size(self) -> int:
        return lib().gsvk_sv_embedding_size(self.h)

    def forward(self, fbank, emb=None, stream=None):
        import torch

        if emb is None:
            emb = torch.empty(self.embedding_size(), device=fbank.device)
        check(lib().gsvk_sv_forward(self.h, _ptr(fbank), fbank.shape[0], _ptr(emb),
                                    _stream(stream)))
        return emb

    def close(self):
        if self.h:
            lib().gsvk_sv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GsvFile:
    """A GSV1 weight container opened through gsvk_gsv_open (host memory)."""

    def __init__(self, path: str):
        h = c_void_p()
        check(lib().gsvk_gsv_open(os.fsencode(path), ctypes.byref(h)))
        self.h = h

    def __len__(self):
        return lib().gsvk_gsv_count(self.h)

    @property
    def model_name(self) -> str:
        return lib().gsvk_gsv_model_name(self.h).decode()

    @property
    def config(self) -> str:
        n = ctypes.c_size_t()
        return lib().gsvk_gsv_config(self.h, ctypes.byref(n)).decode()

    def _arrays(self, t):
        import numpy as np

        shape = tuple(t.dims[:t.rank])
        f32 = f16 = None
        if t.f32:
            f32 = np.ctypeslib.as_array(ctypes.cast(t.f32, ctypes.POINTER(c_float)),
                                        shape=(t.numel,)).reshape(shape).copy()
        if t.f16:
            f16 = np.ctypeslib.as_array(ctypes.cast(t.f16, ctypes.POINTER(ctypes.c_uint16)),
                                        shape=(t.numel,)).reshape(shape).copy()
        return t.name.decode(), shape, t.src_dtype, f32, f16

    def tensor(self, name: str):
        """(name, shape, src_dtype, fp32 array or None, fp16 bits or None)."""
        t = GsvTensor()
        check(lib().gsvk_gsv_find(self.h, name.encode(), ctypes.byref(t)))
        return self._arrays(t)

    def tensors(self):
        out = []
        for i in range(len(self)):
            t = GsvTensor()
            check(lib().gsvk_gsv_tensor_at(self.h, i, ctypes.byref(t)))
            out.append(self._arrays(t))
        return out

    def close(self):
        if self.h:
            lib().gsvk_gsv_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class T2SSampling(ctypes.Structure):
    _fields_ = [("mode", c_int), ("top_k", c_int), ("top_p", c_float), ("temperature", c_float),
                ("rep_penalty", c_float), ("seed", ctypes.c_ulonglong)]


class T2S:
    """Device T2S engine (ar::T2SEngine).  `model` is a dict of numpy arrays in
    the reference layouts (see workloads.t2s_model)."""

    @classmethod
    def from_gsv(cls, gsv: "GsvFile", cap: int):
        """T2SEngine(const GsvFile&) on the device (gsvk_t2s_create_from_gsv)."""
        import json

        self = cls.__new__(cls)
        mc = json.loads(gsv.config)["model_config"]["model"]
        self.model = dict(n_layers=int(mc["n_layer"]), d_model=int(mc["hidden_dim"]),
                          vocab=int(mc["vocab_size"]))
        self._keep = {}
        h = c_void_p()
        check(lib().gsvk_t2s_create_from_gsv(gsv.h, cap, ctypes.byref(h)))
        self.h = h
        self.cap = cap
        return self

    def __init__(self, model: dict, cap: int):
        import numpy as np

        self.model = model
        self.cap = cap
        self._keep = {k: np.ascontiguousarray(v) for k, v in model.items()
                      if isinstance(v, np.ndarray)}
        cfg = T2SConfig(model["n_layers"], model["d_model"], model["n_heads"], model["ffn"],
                        model["vocab"], model["ln_eps"], model["alpha_audio"], cap)
        w = T2SHostWeights(*[self._keep[n].ctypes.data for n in (
            "wqkv", "bqkv", "wout", "bout", "w1", "b1", "w2", "b2", "n1g", "n1b", "n2g", "n2b",
            "wpred", "audio_emb")])
        h = c_void_p()
        check(lib().gsvk_t2s_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().gsvk_t2s_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_kv(self, k, v, prefix: int, stream=None):
        """k, v: host uint16 [L, rows, D] (pinned torch tensors or numpy)."""
        rows = k.shape[1]
        kp = k.ctypes.data if hasattr(k, "ctypes") else k.data_ptr()
        vp = v.ctypes.data if hasattr(v, "ctypes") else v.data_ptr()
        check(lib().gsvk_t2s_load_kv(self.h, kp, vp, prefix, rows, _stream(stream)))

    def prefill(self, x, pos: int, text_len: int = 0, stream=None):
        check(lib().gsvk_t2s_prefill(self.h, _ptr(x), x.shape[0], pos, text_len, _stream(stream)))
        return x

    def generate(self, prefix: int, prompt, max_steps: int, stop_on_eos: bool = True,
                 stream=None):
        """Host prompt (int32 numpy) -> (tokens, margins) numpy arrays."""
        import numpy as np

        pr = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(max(1, max_steps), np.int32)
        margins = np.zeros(max(1, max_steps), np.float32)
        n = c_int(0)
        check(lib().gsvk_t2s_generate(self.h, prefix, pr.ctypes.data, pr.size, max_steps,
                                      int(stop_on_eos), toks.ctypes.data, margins.ctypes.data,
                                      ctypes.byref(n), _stream(stream)))
        return toks[:n.value], margins[:max_steps]

    def generate_device(self, prefix: int, prompt_dev, max_steps: int, tokens_dev, n_out_dev,
                        stop_on_eos: bool = True, margins_dev=None, stream=None):
        check(lib().gsvk_t2s_generate_device(self.h, prefix, _ptr(prompt_dev), prompt_dev.numel(),
                                             max_steps, int(stop_on_eos), _ptr(tokens_dev),
                                             _ptr(n_out_dev), _ptr(margins_dev), _stream(stream)))

    def prompt(self, prefix: int, prompt_dev, stream=None):
        check(lib().gsvk_t2s_prompt(self.h, prefix, _ptr(prompt_dev), prompt_dev.numel(),
                                    _stream(stream)))

    def decode(self, prefix: int, prompt_dev, max_steps: int, tokens_dev, n_out_dev,
               stop_on_eos: bool = True, margins_dev=None, stream=None):
        check(lib().gsvk_t2s_decode(self.h, prefix, _ptr(prompt_dev), prompt_dev.numel(),
                                    max_steps, int(stop_on_eos), _ptr(tokens_dev), _ptr(n_out_dev),
                                    _ptr(margins_dev), _stream(stream)))

    DECODE_GRID, DECODE_CLUSTER, DECODE_FLOW = 1, 2, 3

    def set_decode_kernel(self, kind: int):
        """1 (or 0, the default): grid kernel (one CTA per SM, grid barriers,
        phase trace); 2: single-cluster kernel (raises if unsupported).
        Both give identical tokens, margins, logits and KV."""
        check(lib().gsvk_t2s_set_decode_kernel(self.h, int(kind)))

    def set_sampling(self, mode=1, top_k=15, top_p=1.0, temperature=1.0, rep_penalty=1.35,
                     seed=1):
        """gsvk_t2s_set_sampling; mode 0 (or None) restores greedy."""
        if mode is None or mode == 0:
            check(lib().gsvk_t2s_set_sampling(self.h, None))
            return
        sp = T2SSampling(mode, top_k, top_p, temperature, rep_penalty, seed)
        check(lib().gsvk_t2s_set_sampling(self.h, ctypes.byref(sp)))

    def decode_kernel(self) -> int:
        return lib().gsvk_t2s_decode_kernel(self.h)

    def set_decode_ctas(self, ctas: int):
        """CTAs of the grid decode kernel (0 = one per SM)."""
        check(lib().gsvk_t2s_set_decode_ctas(self.h, int(ctas)))

    def read_kv(self):
        """(k, v) host uint16 [n_layers, cap, d_model]."""
        import numpy as np

        shape = (self.model["n_layers"], self.cap, self.model["d_model"])
        k, v = np.zeros(shape, np.uint16), np.zeros(shape, np.uint16)
        check(lib().gsvk_t2s_read_kv(self.h, k.ctypes.data, v.ctypes.data))
        return k, v

    TRACE_STEPS, TRACE_STRIDE = 4, 16 + 16 * 64

    def set_trace(self, on: bool = True):
        check(lib().gsvk_t2s_set_trace(self.h, int(on)))

    def read_trace(self):
        """[4, 1040] device-clock ns per phase boundary (see gsvk.h)."""
        import numpy as np

        out = np.zeros(self.TRACE_STEPS * self.TRACE_STRIDE, np.uint64)
        check(lib().gsvk_t2s_read_trace(self.h, out.ctypes.data, out.size))
        return out.reshape(self.TRACE_STEPS, self.TRACE_STRIDE)

    def launches_per_generate(self) -> int:
        return lib().gsvk_t2s_launches_per_generate(self.h)

    def read_logits(self):
        import numpy as np

        out = np.zeros(self.model["vocab"], np.float32)
        check(lib().gsvk_t2s_read_logits(self.h, out.ctypes.data))
        return out


# ---------------------------------------------------------- a12 - a15: SoVITS
class ConvArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("T", _sz), ("ci", _sz), ("w", _vp), ("co", _sz), ("k", _sz),
                ("dil", _sz), ("bias", _vp), ("residual", _vp), ("res_scale", c_float),
                ("act", c_int), ("slope", c_float), ("y", _vp), ("y_f16", _vp),
                ("y_f16_act", _vp), ("act2", c_int), ("slope2", c_float)]


def pack_conv_weight(w_torch, transpose=False, stream=None):
    """fp16 torch-layout weight (CUDA) -> packed [k][co][ci]."""
    import torch

    if transpose:
        ci, co, k = w_torch.shape
    else:
        co, ci, k = w_torch.shape
    out = torch.empty(k, co, ci, dtype=torch.float16, device=w_torch.device)
    fn = lib().gsvk_convt1d_pack_weight if transpose else lib().gsvk_conv1d_pack_weight
    a, b = (ci, co) if transpose else (co, ci)
    check(fn(_ptr(w_torch), a, b, k, _ptr(out), _stream(stream)))
    return out


def conv1d(x16, wp, bias=None, dil=1, transpose=False, residual=None, res_scale=1.0,
           act=ACT_NONE, slope=0.0, y=None, y_f16=None, y_f16_act=None, act2=ACT_NONE,
           slope2=0.0, stream=None):
    """Channels-last conv (x16 [T, ci] fp16, wp packed [k, co, ci]); transpose=True
    runs ConvTranspose1d with stride `dil`."""
    import torch

    T, ci = x16.shape
    k, co, ci2 = wp.shape
    assert ci == ci2
    t_out = T * dil if transpose else T
    if y is None and y_f16 is None and y_f16_act is None:
        y = torch.empty(t_out, co, device=x16.device)
    a = ConvArgs(_ptr(x16), T, ci, _ptr(wp), co, k, dil, _ptr(bias), _ptr(residual), res_scale,
                 act, slope, _ptr(y), _ptr(y_f16), _ptr(y_f16_act), act2, slope2)
    fn = lib().gsvk_convt1d_f16 if transpose else lib().gsvk_conv1d_f16
    check(fn(ctypes.byref(a), _stream(stream)))
    return y


def channels_to_rows_f16(x, stream=None):
    import torch

    C, T = x.shape
    y = torch.empty(T, C, dtype=torch.float16, device=x.device)
    check(lib().gsvk_channels_to_rows_f16(_ptr(x), C, T, _ptr(y), _stream(stream)))
    return y


def rows_to_channels_f32(x, stream=None):
    import torch

    T, C = x.shape
    y = torch.empty(C, T, device=x.device)
    check(lib().gsvk_rows_to_channels_f32(_ptr(x), T, C, _ptr(y), _stream(stream)))
    return y


class DecoderConfig(ctypes.Structure):
    _fields_ = [("n_stages", c_int), ("in_ch", c_int), ("ch0", c_int), ("conv_pre_k", c_int),
                ("conv_post_k", c_int), ("up_rate", c_int * 8), ("up_k", c_int * 8),
                ("res_k", c_int * 3), ("res_dil", c_int * 3), ("lrelu_slope", c_float),
                ("post_slope", c_float), ("max_frames", c_int)]


class Decoder:
    """Device HiFi-GAN generator (sovits::Generator).  ws/bs: host numpy weights
    in the documented order (workloads.decoder_weights)."""

    def __init__(self, cfg: dict, ws, bs, max_frames: int):
        import numpy as np

        c = DecoderConfig()
        c.n_stages, c.in_ch, c.ch0 = cfg["n_stages"], cfg["in_ch"], cfg["ch0"]
        c.conv_pre_k, c.conv_post_k = cfg["conv_pre_k"], cfg["conv_post_k"]
        for i in range(cfg["n_stages"]):
            c.up_rate[i], c.up_k[i] = cfg["up_rate"][i], cfg["up_k"][i]
        for i in range(3):
            c.res_k[i], c.res_dil[i] = cfg["res_k"][i], cfg["res_dil"][i]
        c.lrelu_slope, c.post_slope, c.max_frames = cfg["lrelu_slope"], cfg["post_slope"], max_frames
        self.cfg = c
        self._ws = [np.ascontiguousarray(w) for w in ws]
        self._bs = [None if b is None else np.ascontiguousarray(b, np.float32) for b in bs]
        wp = (c_void_p * len(ws))(*[w.ctypes.data for w in self._ws])
        bp = (c_void_p * len(bs))(*[None if b is None else b.ctypes.data for b in self._bs])
        h = c_void_p()
        check(lib().gsvk_decoder_create(ctypes.byref(c), wp, bp, ctypes.byref(h)))
        self.h = h

    def out_len(self, T: int) -> int:
        return lib().gsvk_decoder_out_len(ctypes.byref(self.cfg), T)

    def forward(self, z, wav=None, stream=None):
        """z: CUDA fp32 [in_ch, T] -> wav CUDA fp32 [T * prod(up_rate)]."""
        import torch

        T = z.shape[1]
        wav = wav if wav is not None else torch.empty(self.out_len(T), device=z.device)
        check(lib().gsvk_decoder_forward(self.h, _ptr(z), T, _ptr(wav), _stream(stream)))
        return wav

    def launches(self) -> int:
        return lib().gsvk_decoder_launches(self.h)

    def set_graph(self, enable: bool):
        """Replay the layers as one CUDA graph per input length (default) or
        launch them one by one; the results are identical."""
        check(lib().gsvk_decoder_set_graph(self.h, int(bool(enable))))

    def close(self):
        if self.h:
            lib().gsvk_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------ a20, a21: encoders
class EncoderConfig(ctypes.Structure):
    _fields_ = [("layers", c_int), ("hidden", c_int), ("heads", c_int), ("ffn", c_int),
                ("eps", c_double), ("max_batch", c_int), ("max_seq", c_int)]


class EncoderHostWeights(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("wqkv", "bqkv", "wo", "bo", "ln1g", "ln1b", "wi", "bi", "wf",
                                   "bf", "ln2g", "ln2b")]


class Encoder:
    """Device encoder stack (BERT / HuBERT); model from workloads.encoder_model."""

    NAMES = ("wqkv", "bqkv", "wo", "bo", "ln1g", "ln1b", "wi", "bi", "wf", "bf", "ln2g", "ln2b")

    def __init__(self, model: dict, max_batch: int, max_seq: int):
        import numpy as np

        self._keep = {n: np.ascontiguousarray(model[n]) for n in self.NAMES}
        cfg = EncoderConfig(model["layers"], model["hidden"], model["heads"], model["ffn"],
                            model["eps"], max_batch, max_seq)
        w = EncoderHostWeights(*[self._keep[n].ctypes.data for n in self.NAMES])
        h = c_void_p()
        check(lib().gsvk_encoder_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(h)))
        self.h = h

    def forward(self, x, batch: int, seq: int, valid=None, stream=None):
        """x: CUDA fp32 [batch*seq, hidden], updated in place."""
        check(lib().gsvk_encoder_forward(self.h, _ptr(x), batch, seq, _ptr(valid),
                                         _stream(stream)))
        return x

    def launches(self) -> int:
        return lib().gsvk_encoder_launches(self.h)

    def close(self):
        if self.h:
            lib().gsvk_encoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------- config 3: batched T2S
class T2SBatch:
    """Batched greedy decode of concurrent utterances (gsvk_t2s_batch_*)."""

    def __init__(self, model: dict, cap: int, max_batch: int, max_steps: int):
        import numpy as np

        self.model = model
        self._keep = {k: np.ascontiguousarray(v) for k, v in model.items()
                      if isinstance(v, np.ndarray)}
        cfg = T2SConfig(model["n_layers"], model["d_model"], model["n_heads"], model["ffn"],
                        model["vocab"], model["ln_eps"], model["alpha_audio"], cap)
        w = T2SHostWeights(*[self._keep[n].ctypes.data for n in (
            "wqkv", "bqkv", "wout", "bout", "w1", "b1", "w2", "b2", "n1g", "n1b", "n2g", "n2b",
            "wpred", "audio_emb")])
        h = c_void_p()
        check(lib().gsvk_t2s_batch_create(ctypes.byref(cfg), ctypes.byref(w), max_batch,
                                          max_steps, ctypes.byref(h)))
        self.h = h
        self.B = 0

    def load_kv(self, b: int, k, v, length: int, stream=None):
        """k, v: [L, rows, D] fp16 bits, numpy (host) or torch (host or CUDA)."""
        kp = k.ctypes.data if hasattr(k, "ctypes") else k.data_ptr()
        vp = v.ctypes.data if hasattr(v, "ctypes") else v.data_ptr()
        check(lib().gsvk_t2s_batch_load_kv(self.h, b, kp, vp, length, k.shape[1],
                                           _stream(stream)))

    def begin(self, lengths, pe0, first_tok, hist=None, stream=None):
        import numpy as np

        B = len(lengths)
        ln = np.ascontiguousarray(lengths, np.int32)
        pe = np.ascontiguousarray(pe0, np.int32)
        ft = np.ascontiguousarray(first_tok, np.int32)
        hs = None if hist is None else np.ascontiguousarray(hist, np.int32)
        check(lib().gsvk_t2s_batch_begin(self.h, B, ln.ctypes.data, pe.ctypes.data, ft.ctypes.data,
                                         None if hs is None else hs.ctypes.data,
                                         0 if hs is None else hs.shape[1], _stream(stream)))
        self.B = B

    def run(self, steps: int, use_graph: bool = True, stream=None):
        check(lib().gsvk_t2s_batch_run(self.h, steps, int(use_graph), _stream(stream)))

    def read(self, steps: int):
        import numpy as np

        toks = np.zeros((steps, self.B), np.int32)
        marg = np.zeros((steps, self.B), np.float32)
        check(lib().gsvk_t2s_batch_read(self.h, steps, toks.ctypes.data, marg.ctypes.data))
        return toks, marg

    ATTN_CHUNK, ATTN_STREAM = 0, 1

    def set_attention(self, kind: int):
        """Attention kernel of the step (ATTN_CHUNK / ATTN_STREAM)."""
        check(lib().gsvk_t2s_batch_set_attention(self.h, int(kind)))

    def attention(self) -> int:
        return lib().gsvk_t2s_batch_attention(self.h)

    def read_logits(self):
        import numpy as np

        out = np.zeros((self.B, self.model["vocab"]), np.float32)
        check(lib().gsvk_t2s_batch_read_logits(self.h, out.ctypes.data))
        return out

    def launches_per_step(self) -> int:
        return lib().gsvk_t2s_batch_launches_per_step(self.h)

    def close(self):
        if self.h:
            lib().gsvk_t2s_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
