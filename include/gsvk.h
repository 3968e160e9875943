/* gsvk.h — C ABI of the B200 (sm_100a) build of the GPT-SoVITS-native
 * `src/kern` GEMM/GEMV hot path and of its callers' fused steps.
 *
 * Conventions (shared by every entry point):
 *  - All tensor pointers are DEVICE pointers unless a parameter says "host".
 *    fp16 values are IEEE binary16 bit patterns in uint16_t, exactly like the
 *    reference's `const uint16_t*` weights.  Matrices are row-major.
 *  - Outputs are overwritten, never accumulated (accel.hpp:68, beta = 0).
 *  - Every call is asynchronous on `stream` (NULL = legacy default stream)
 *    and returns a status: 0 = ok, negative = error (see GSVK_ERR_*).  The
 *    reference returns silently on invalid shapes (gemm_f16_amx.cpp:551-553);
 *    this ABI reports them instead and writes nothing.
 *  - No call allocates device memory on the hot path.  Workspaces are
 *    created by the *_create entry points and owned by their handles.
 *  - Thread-safe per stream: calls on different streams may run
 *    concurrently; a handle must not be used from two streams at once.
 *
 * gsvk_stream_t is ABI-compatible with cudaStream_t / CUstream.
 */
#ifndef GSVK_H
#define GSVK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gsvk_stream_t;

enum {
  GSVK_OK = 0,
  GSVK_ERR_INVALID = -1,     /* null pointer, zero or inconsistent size */
  GSVK_ERR_ALIGN = -2,       /* pointer or leading dimension misaligned */
  GSVK_ERR_CUDA = -3,        /* CUDA runtime / driver error */
  GSVK_ERR_TIMEOUT = -4,     /* a bounded device-side wait gave up */
  GSVK_ERR_UNSUPPORTED = -5, /* shape outside the kernel's envelope */
  GSVK_ERR_NOMEM = -6,       /* a *_create entry point could not allocate */
  GSVK_ERR_NODEV = -7        /* no sm_100 device */
};

/* Epilogue activation codes (y = act(acc + bias) [+ residual]). */
enum {
  GSVK_ACT_NONE = 0,
  GSVK_ACT_RELU = 1,     /* kern.cpp:85 relu */
  GSVK_ACT_GELU_ERF = 2, /* bert_ops.hpp:25 gelu_erf */
  GSVK_ACT_LEAKY = 3     /* nn_ops.hpp:48 leaky_relu(slope) */
};

/* ---- library ---------------------------------------------------------- */
int gsvk_version(void);
/* Human-readable text of the last error raised on the calling thread. */
const char* gsvk_last_error(void);
/* Selects `device` for the calling thread, checks it is sm_100, and resolves
 * the driver entry points the TMA paths need.  Replaces the reference's
 * availability probe kern::amx_gemm_available() (gemm_f16_amx.hpp:32). */
int gsvk_device_init(int device);
/* 1 when gsvk_device_init succeeded on the current device. */
int gsvk_available(void);
/* Reads (and optionally clears) the current device's status word written by
 * bounded device-side waits; synchronous.  GSVK_ERR_TIMEOUT when a kernel
 * gave up waiting since the last reset. */
int gsvk_device_status(int reset);

/* ---- fp16 conversion (a4) ---------------------------------------------- */
/* kern::f32_to_f16 (gemv_fmlal.hpp:16): round-to-nearest-even. */
int gsvk_f32_to_f16(const float* src, uint16_t* dst, size_t n, gsvk_stream_t stream);
/* accel::f16_to_f32 (accel.hpp:33): exact widening. */
int gsvk_f16_to_f32(const uint16_t* src, float* dst, size_t n, gsvk_stream_t stream);

/* ---- decode GEMV (a1, a2) ---------------------------------------------- */
/* kern::gemv_f16w_f32acc (kern.hpp:15): y[out] = W[out,in] . x[in];
 * W fp16, x and y fp32, fp32 accumulation. */
int gsvk_gemv_f16w_f32acc(const uint16_t* w, const float* x, float* y, size_t out,
                          size_t in, gsvk_stream_t stream);
/* kern::gemv_f16x_fmlal (gemv_fmlal.hpp:26): fp16 x, products exact in fp32. */
int gsvk_gemv_f16x_fmlal(const uint16_t* w, const uint16_t* xh, float* y, size_t out,
                         size_t in, gsvk_stream_t stream);
/* Fused form used by the callers' decode steps (t2s_engine.cpp:1044-1118):
 *   y = act(W.x + bias) + residual
 * x is fp16 when x_is_f16 != 0, else fp32; bias/residual may be NULL;
 * y_f16 (optional) receives the same values rounded to fp16. */
int gsvk_gemv_ex(const uint16_t* w, const void* x, int x_is_f16, float* y, uint16_t* y_f16,
                 size_t out, size_t in, const float* bias, const float* residual, int act,
                 float slope, gsvk_stream_t stream);

/* ---- tensor-core GEMM (a3, a6, a9) -------------------------------------- */
/* kern::gemm_f16x_fmlal (gemv_fmlal.hpp:36): C[M,N] = A[M,K] . B[N,K]^T,
 * fp16 A/B row-major, fp32 C row-major.  tcgen05 + TMA when K and the
 * leading dimensions are multiples of 8 (16-byte rows), a CUDA-core kernel
 * otherwise (same results within fp32 rounding). */
int gsvk_gemm_f16(const uint16_t* a, const uint16_t* b, float* c, size_t M, size_t N, size_t K,
                  gsvk_stream_t stream);

/* Fused form: C = act(alpha * A.B^T + bias) + residual, written as fp32
 * and/or fp16.  Covers accel::DenseF16::forward on a view (accel.hpp:70-78)
 * and bert::Linear::forward (bert_ops.hpp:225-258) with their bias / GELU /
 * residual loops folded into the epilogue.  Zero leading dimensions mean
 * "dense" (K for A/B, N for C / residual). */
typedef struct {
  const uint16_t* a; size_t lda;     /* [M, K] fp16 */
  const uint16_t* b; size_t ldb;     /* [N, K] fp16 (weights, [out, in]) */
  size_t M, N, K;
  const float* bias;                 /* [N] or NULL */
  const float* residual; size_t ld_res; /* fp32 [M, N] or NULL */
  float* c; size_t ldc;              /* fp32 output or NULL */
  uint16_t* c_f16; size_t ldc_f16;   /* fp16 output or NULL */
  int act; float slope;              /* GSVK_ACT_* */
  float alpha;                       /* 0 is read as 1 */
} gsvk_gemm_args;
int gsvk_gemm_f16_ex(const gsvk_gemm_args* args, gsvk_stream_t stream);

/* ---- support primitives (a22) ------------------------------------------ */
/* kern::layernorm (kern.cpp:27) applied to `rows` rows of n. y may equal x. */
int gsvk_layernorm_rows(const float* x, const float* g, const float* b, float* y,
                        size_t rows, size_t n, double eps, gsvk_stream_t stream);
/* kern::softmax_rows (kern.cpp:76). */
int gsvk_softmax_rows(const float* x, float* y, size_t rows, size_t n,
                      gsvk_stream_t stream);
/* relu / gelu_erf / leaky_relu(slope) elementwise, fp32. */
int gsvk_activation(const float* x, float* y, size_t n, int act, float slope,
                    gsvk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
