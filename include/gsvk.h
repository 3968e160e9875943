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
  GSVK_ACT_LEAKY = 3,    /* nn_ops.hpp:48 leaky_relu(slope) */
  GSVK_ACT_TANH = 4      /* dec.hpp:344 output tanh */
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
/* Plain GEMMs with M, N >= 256 and K a multiple of 64 (here and in the
 * engines built on this library) may run on the two-SM kernel (256 x 256
 * tiles over a CTA pair, tcgen05.mma.cta_group::2).  mode 1 (the default):
 * when its tile rounds cost no more than the one-SM kernel's; 2: always;
 * 0: never.  Process-wide; GSVK_ERR_INVALID for another mode. */
int gsvk_gemm_set_pair(int mode);
/* 1 if gsvk_gemm_f16_ex of an M x N x K problem (16-byte aligned operands,
 * leading dimensions K) runs on the two-SM kernel under the current mode,
 * 0 otherwise.  A query only: launches nothing. */
int gsvk_gemm_uses_pair(size_t M, size_t N, size_t K);
/* enable != 0 (the default): the one-SM tensor-core kernel (convolutions and
 * the GEMMs kept off the two-SM kernel) writes its fp32 / fp16 / activated
 * fp16 outputs through shared-memory tiles and TMA bulk stores where the
 * problem allows (contiguous output rows, 16-byte aligned outputs, no
 * transposed-V output); 0: per-row stores everywhere.
 * Results are identical either way.  Process-wide. */
int gsvk_gemm_set_bulk_epilogue(int enable);

/* Strided batched GEMM: `batch` independent problems of one shape and one
 * epilogue, problem i reading A at args->a + i*stride_a and B at
 * args->b + i*stride_b (stride_b = 0: shared weights) and writing C (and the
 * residual it reads) at + i*stride_c; strides in elements.  When the strides
 * are whole rows of their tensors (stride % leading dimension == 0) and the
 * outputs share one row layout, all problems run as ONE persistent
 * tensor-core launch over every (problem, tile); otherwise one launch per
 * problem.  The batched form of AmxBatchNode / amx_batch_run for
 * same-shape work (gemm_f16_amx.hpp:64-78). */
int gsvk_gemm_f16_batched(const gsvk_gemm_args* args, size_t batch, size_t stride_a,
                          size_t stride_b, size_t stride_c, gsvk_stream_t stream);

/* Grouped GEMM: `count` independent problems (each with its own operands,
 * shapes and epilogue) submitted together on one stream, in order.  Replaces
 * AmxBatchNode + amx_batch_run (gemm_f16_amx.hpp:64-78).  Every group is
 * validated before any is launched. */
int gsvk_gemm_grouped_f16(const gsvk_gemm_args* groups, size_t count, gsvk_stream_t stream);

/* Chained GEMMs: the analogue of AmxChainLink + amx_chain_run and
 * AmxTileChainLink + amx_tile_chain_run (gemm_f16_amx.hpp:90-124).  Links of
 * one chain_id run in depth order (depth d after depth d - 1, so a link may
 * read the output of the link before it); links of different chains are
 * independent.  Each link computes exactly what gsvk_gemm_f16_ex computes
 * for its arguments.  The reference's host-side `prepare` hook (im2col into
 * a packed panel) has no counterpart: a link's operands are device tensors
 * the previous link's epilogue writes directly (convolutions take their
 * taps by TMA coordinate shifts, gsvk_conv1d_f16).  Depths 0..4095; a
 * repeated (chain_id, depth) pair or an invalid GEMM fails before anything
 * is launched.  Work is queued on `stream` level by level. */
typedef struct {
  int chain_id;
  int depth;
  gsvk_gemm_args gemm;
} gsvk_gemm_chain_link;
int gsvk_gemm_chain_run(const gsvk_gemm_chain_link* links, size_t n, gsvk_stream_t stream);

/* ---- weight registration (a8) ------------------------------------------- */
/* The analogue of amx_pack / AmxPanel (gemm_f16_amx.hpp:36-50): a one-off
 * load-time upload of a row-major [rows, cols] fp16 weight (host or device
 * memory) into a device copy the handle owns.  The row-major layout is what
 * the TMA descriptors read, so no re-packing happens. */
typedef struct gsvk_weights* gsvk_weights_t;
int gsvk_weights_register(const uint16_t* w, size_t rows, size_t cols, gsvk_weights_t* out);
int gsvk_weights_release(gsvk_weights_t w);
const uint16_t* gsvk_weights_data(gsvk_weights_t w); /* device pointer, [rows, cols] */
/* gsvk_gemm_f16_ex with B taken from the handle (args->b / ldb ignored;
 * args->N, K must equal rows, cols). */
int gsvk_gemm_f16_w(const gsvk_gemm_args* args, gsvk_weights_t w, gsvk_stream_t stream);
/* gsvk_gemv_f16w_f32acc over a registered [out, in] weight. */
int gsvk_gemv_f16w_f32acc_w(gsvk_weights_t w, const float* x, float* y, gsvk_stream_t stream);

/* ---- fp32 GEMM (a5) ------------------------------------------------------ */
/* accel::sgemm (accel.hpp:27): row-major C = alpha op(A) op(B) + beta C with
 * transa/transb 'N' or 'T'; beta == 0 never reads C.  fp32 on CUDA cores. */
int gsvk_sgemm(char transa, char transb, int M, int N, int K, float alpha, const float* A,
               int lda, const float* B, int ldb, float beta, float* C, int ldc,
               gsvk_stream_t stream);

/* accel::gemm_nt_f16w (accel.hpp:38-41): y[T, out] = x[T, in] . W[out, in]^T
 * with fp32 activations and fp16 weights widened exactly, one fp32 FMA chain
 * per output in k order on CUDA cores -- bit-identical to gsvk_sgemm on an
 * fp32 up-cast copy of W (which is how the reference computes it, and how
 * its resident DenseF16 forward runs, accel.hpp:85-92).  Device pointers. */
int gsvk_gemm_nt_f16w(const float* x, size_t T, size_t in, const uint16_t* w, size_t out,
                      float* y, gsvk_stream_t stream);

/* Device buffers for host code that does not link the CUDA runtime (the
 * C++ shim's resident DenseF16 keeps its fp32 weights in one): allocates
 * `bytes` of device memory and fills it from `src` (host or device memory),
 * or with zeros when src is NULL.  Load-time helpers, not for the hot path. */
int gsvk_device_alloc_copy(const void* src, size_t bytes, void** out);
int gsvk_device_free(void* p);

/* ---- SoVITS convolutions (a12-a14) -------------------------------------- */
/* Activations are channels-last rows: x[T][ci] fp16 (the transpose of the
 * reference's channel-major Tensor2D, sovits_types.hpp), ci a multiple of 8.
 * Weights are packed once to tap-major [k][co][ci] fp16 by the pack entry
 * points below (the reference's ConvT phase layout, conv1d.hpp:226-232).
 * The epilogue writes y = act(conv + bias) + res_scale * residual as fp32
 * (y), fp16 (y_f16) and/or fp16 of act2(y) (y_f16_act), all [T_out][co]. */
typedef struct {
  const uint16_t* x; size_t T; size_t ci;
  const uint16_t* w; size_t co; size_t k;
  size_t dil;              /* conv1d: dilation (1 = plain); convt1d: stride u */
  const float* bias;       /* [co] or NULL */
  const float* residual;   /* fp32 [T_out][co] or NULL (may alias y) */
  float res_scale;
  int act; float slope;
  float* y; uint16_t* y_f16; uint16_t* y_f16_act;
  int act2; float slope2;
} gsvk_conv_args;
/* torch Conv1d weight [co][ci][k] -> packed [k][co][ci] (DEVICE buffers). */
int gsvk_conv1d_pack_weight(const uint16_t* w_torch, size_t co, size_t ci, size_t k,
                            uint16_t* packed, gsvk_stream_t stream);
/* torch ConvTranspose1d weight [ci][co][k] -> packed [k][co][ci]. */
int gsvk_convt1d_pack_weight(const uint16_t* w_torch, size_t ci, size_t co, size_t k,
                             uint16_t* packed, gsvk_stream_t stream);
/* sovits::Conv1d::forward (conv1d.hpp:109-194): same padding (k-1)*dil/2,
 * implicit GEMM on the tensor cores (no im2col buffer); T_out = T. */
int gsvk_conv1d_f16(const gsvk_conv_args* args, gsvk_stream_t stream);
/* sovits::ConvT1d::forward (conv1d.hpp:250-359): ConvTranspose1d(k, stride u,
 * pad (k-u)/2), polyphase implicit GEMM writing every output phase directly;
 * T_out = T * u.  Requires k >= u and k - u even. */
int gsvk_convt1d_f16(const gsvk_conv_args* args, gsvk_stream_t stream);
/* Layout helpers: channel-major fp32 [C][T] <-> channels-last rows. */
int gsvk_channels_to_rows_f16(const float* x, size_t C, size_t T, uint16_t* y,
                              gsvk_stream_t stream);
int gsvk_rows_to_channels_f32(const float* x, size_t T, size_t C, float* y, gsvk_stream_t stream);

/* ---- SoVITS HiFi-GAN generator (a15) ------------------------------------ */
/* sovits::Generator::forward (dec.hpp:265-345) without the cond(ge) term:
 * conv_pre -> n_stages x [lrelu -> ConvT -> mean of 3 ResBlock1] -> lrelu
 * (post_slope) -> conv_post -> tanh.  Weights (HOST, torch layouts, fp16)
 * in the order: [0] conv_pre; per stage s: [1+19s] ups[s], then resblock j
 * pair p: [1+19s+1+6j+2p] convs1[p], [+1] convs2[p]; [1+19*n_stages]
 * conv_post.  Biases fp32 (NULL allowed).  max_frames bounds T. */
typedef struct gsvk_decoder* gsvk_decoder_t;
typedef struct {
  int n_stages, in_ch, ch0, conv_pre_k, conv_post_k;
  int up_rate[8], up_k[8];
  int res_k[3], res_dil[3];
  float lrelu_slope, post_slope;
  int max_frames;
} gsvk_decoder_config;
size_t gsvk_decoder_out_len(const gsvk_decoder_config* cfg, size_t T);
int gsvk_decoder_create(const gsvk_decoder_config* cfg, const uint16_t* const* w_host,
                        const float* const* b_host, gsvk_decoder_t* out);
int gsvk_decoder_destroy(gsvk_decoder_t h);
/* z: DEVICE fp32 [in_ch][T] (channel-major, the reference layout);
 * wav: DEVICE fp32 [T * prod(up_rate)]. */
int gsvk_decoder_forward(gsvk_decoder_t h, const float* z, size_t T, float* wav,
                         gsvk_stream_t stream);
/* Kernel launches issued by the last gsvk_decoder_forward. */
int gsvk_decoder_launches(gsvk_decoder_t h);
/* enable != 0 (the default): the layers between conv_pre's input and
 * conv_post are captured once per input length T into a CUDA graph and
 * replayed; 0: they are launched one by one.  The results are identical. */
int gsvk_decoder_set_graph(gsvk_decoder_t h, int enable);

/* ---- encoder stacks: RoBERTa-large / HuBERT-base (a20, a21) -------------- */
/* bert::BertLayer::forward (bert_ops.hpp:347-400) and the HuBERT layer loop
 * (hubert.cpp:590-730), post-LN, GELU(erf) FFN, every product on the tensor
 * cores (q/k/v fused into one GEMM, attention as batched GEMMs).  HOST
 * weights: fp16 [L][3C][C] (q, k, v rows), [L][C][C], [L][F][C], [L][C][F];
 * fp32 biases and LayerNorm parameters.  hidden, ffn and head_dim must be
 * multiples of 64; seq <= 256. */
typedef struct gsvk_encoder* gsvk_encoder_t;
typedef struct {
  int layers, hidden, heads, ffn;
  double eps;            /* 1e-12 RoBERTa, 1e-5 HuBERT */
  int max_batch, max_seq;
} gsvk_encoder_config;
typedef struct {
  const uint16_t* wqkv; const float* bqkv;
  const uint16_t* wo;   const float* bo;
  const float* ln1g; const float* ln1b;
  const uint16_t* wi;   const float* bi;
  const uint16_t* wf;   const float* bf;
  const float* ln2g; const float* ln2b;
} gsvk_encoder_host_weights;
int gsvk_encoder_create(const gsvk_encoder_config* cfg, const gsvk_encoder_host_weights* w,
                        gsvk_encoder_t* out);
int gsvk_encoder_destroy(gsvk_encoder_t h);
/* x: DEVICE fp32 [batch*seq][hidden], replaced by the stack's output.
 * valid (DEVICE int32 [batch], optional): keys >= valid[b] are masked with
 * finfo.min as the reference's attention mask (bert_ops.hpp:373-374). */
int gsvk_encoder_forward(gsvk_encoder_t h, float* x, size_t batch, size_t seq, const int* valid,
                         gsvk_stream_t stream);
int gsvk_encoder_launches(gsvk_encoder_t h);

/* ---- HuBERT feature front-end (hubert.cpp:439-580) ---------------------- */
/* The 7-layer strided CNN feature extractor (valid convolutions, no bias;
 * layer 0 with a per-channel GroupNorm: fp64 mean and biased variance over
 * time; GELU after every layer), the feature projection (LayerNorm,
 * Linear + bias on fp16 activations), the grouped positional convolution
 * (pad pos_k/2, the first T of its T + 1 outputs, + bias, GELU, added to the
 * projected features) and the encoder LayerNorm: waveform -> the input of
 * the transformer layers (gsvk_encoder_forward).  Convolutions round their
 * activations to fp16 and accumulate in fp32 on the tensor cores, as the
 * reference's im2col + gemm_f16x_fmlal / AMX path does. */
typedef struct gsvk_hubert_front* gsvk_hubert_front_t;
typedef struct {
  int conv_dim[7];      /* 512 x 7 */
  int conv_kernel[7];   /* 10, 3, 3, 3, 3, 2, 2 */
  int conv_stride[7];   /* 5, 2, 2, 2, 2, 2, 2 */
  int hidden;           /* 768 */
  int pos_k;            /* num_conv_pos_embeddings, 128 */
  int pos_groups;       /* num_conv_pos_embedding_groups, 16 */
  float ln_eps;         /* layer_norm_eps, 1e-5 */
  size_t max_samples;   /* longest waveform a forward may take */
} gsvk_hubert_front_config;
/* HOST pointers, the reference's tensor layouts: conv_w[i] fp16
 * [conv_dim[i]][in][k]; gn_* [conv_dim[0]]; proj_ln_* [conv_dim[6]];
 * proj_w fp16 [hidden][conv_dim[6]], proj_b [hidden]; pos_w fp32
 * [hidden][hidden/pos_groups][pos_k] (the weight-norm product, rounded to
 * fp16 once at create, hubert.cpp:538-539), pos_b [hidden]; enc_ln_* [hidden]. */
typedef struct {
  const uint16_t* conv_w[7];
  const float* gn_g; const float* gn_b;
  const float* proj_ln_g; const float* proj_ln_b;
  const uint16_t* proj_w; const float* proj_b;
  const float* pos_w; const float* pos_b;
  const float* enc_ln_g; const float* enc_ln_b;
} gsvk_hubert_front_weights;
int gsvk_hubert_front_create(const gsvk_hubert_front_config* cfg,
                             const gsvk_hubert_front_weights* w, gsvk_hubert_front_t* out);
int gsvk_hubert_front_destroy(gsvk_hubert_front_t h);
/* Frames the CNN makes of n samples (0 when too short). */
size_t gsvk_hubert_front_frames(gsvk_hubert_front_t h, size_t n);
/* wav: DEVICE fp32 [n]; x: DEVICE fp32 [frames][hidden]. */
int gsvk_hubert_front_forward(gsvk_hubert_front_t h, const float* wav, size_t n, float* x,
                              gsvk_stream_t stream);

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

/* ---- decode attention (a17 support op) ---------------------------------- */
/* The per-head attention of one decode step (t2s_engine.cpp:1062-1087):
 *   out[h] = softmax(q[h] . K[0:len, h]^T * scale) . V[0:len, h]
 * over a token-major fp16 cache whose rows hold row_stride halves (head h at
 * column h*head_dim).  Canonical chunked softmax (64-slot chunks, the T2S
 * decode kernel's order: bit-identical results).  q and out are fp32
 * [n_heads * head_dim]; head_dim 32 or 64.  workspace: DEVICE floats, at least
 * gsvk_attention_workspace_floats(len, n_heads, head_dim) of them. */
size_t gsvk_attention_workspace_floats(size_t len, size_t n_heads, size_t head_dim);
int gsvk_attention_decode(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                          size_t len, size_t n_heads, size_t head_dim, size_t row_stride,
                          float scale, float* out, float* workspace, gsvk_stream_t stream);

/* Allocation-free form of gsvk_attention_decode, for callers that cannot
 * allocate device memory (a host framework whose pool owns all device
 * memory, a fixed-budget deployment, a call path that must not touch the CUDA
 * allocator).  No counterpart in the reference, whose CPU kernels keep their
 * scratch in thread-local vectors.  The chunk records live in one static
 * device array of gsvk_attention_decode_noalloc_max_floats() floats (1 MiB),
 * held by every GPU that loads the library until the process exits; requests
 * needing more (n_heads * ceil(len/64) * (head_dim+4) floats) return
 * GSVK_ERR_UNSUPPORTED.  The first call on a device resolves the array's
 * device address in the current driver context (and a call made from a
 * different context, e.g. after a device reset, resolves it again); make that
 * first call before any stream capture.  All calls
 * on a device share the array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller.  Results
 * are bit-identical to gsvk_attention_decode. */
size_t gsvk_attention_decode_noalloc_max_floats(void);
int gsvk_attention_decode_noalloc(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                  size_t len, size_t n_heads, size_t head_dim, size_t row_stride,
                                  float scale, float* out, gsvk_stream_t stream);

/* ---- T2S autoregressive transformer (a16-a19) -------------------------- */
/* Replaces ar::T2SEngine (t2s_engine.hpp:86-220): weights registered once
 * (the analogue of the reference's load + amx_pack), KV cache and every
 * workspace owned by the handle. */
typedef struct gsvk_t2s* gsvk_t2s_t;
typedef struct {
  int n_layers, d_model, n_heads, ffn, vocab; /* 24, 512, 16, 2048, 1025 */
  float ln_eps;                               /* 1e-5 */
  float alpha_audio;                          /* ar_audio_position.alpha */
  int cap;                                    /* KV slots (prefix + prompt + steps) */
} gsvk_t2s_config;
/* HOST pointers, layouts of the reference's .gsv tensors (t2s_engine.cpp:606-627):
 * fp16 [L][3D][D] in_proj, [L][D][D] out_proj, [L][F][D] linear1,
 * [L][D][F] linear2, [V][D] predict_layer and audio embedding; fp32 biases
 * and LayerNorm affine parameters. */
typedef struct {
  const uint16_t* wqkv; const float* bqkv;
  const uint16_t* wout; const float* bout;
  const uint16_t* w1;   const float* b1;
  const uint16_t* w2;   const float* b2;
  const float* n1g; const float* n1b;
  const float* n2g; const float* n2b;
  const uint16_t* wpred;
  const uint16_t* audio_emb;
} gsvk_t2s_host_weights;
int gsvk_t2s_create(const gsvk_t2s_config* cfg, const gsvk_t2s_host_weights* w, gsvk_t2s_t* out);

/* ---- .gsv weight container (GsvFile, src/runtime/gsv_loader.hpp:50-114;
 * GSV1 format per tools/convert.py:3-28) -------------------------------- */
/* Opens and validates a GSV1 file (mapped read-only; the rules of the
 * reference loader: magic, version, truncation, rank <= 8, known dtype,
 * segment sizes matching the shape, 64-byte aligned in-file segments, flag
 * bit 0 equal to the presence of fp16 segments).  Host-only: needs no GPU. */
typedef struct gsvk_gsv* gsvk_gsv_t;
typedef struct {
  const char* name;
  uint32_t rank;
  uint32_t dims[8];
  int src_dtype;          /* 1 fp32, 2 fp16 (the checkpoint's type) */
  uint64_t numel;
  const float* f32;       /* fp32 copy (host, in the mapping) or NULL (slim fp16-only) */
  const uint16_t* f16;    /* fp16 copy or NULL */
} gsvk_gsv_tensor;
int gsvk_gsv_open(const char* path, gsvk_gsv_t* out);
int gsvk_gsv_close(gsvk_gsv_t f);
size_t gsvk_gsv_count(gsvk_gsv_t f);
const char* gsvk_gsv_model_name(gsvk_gsv_t f);
const char* gsvk_gsv_config(gsvk_gsv_t f, size_t* len); /* the embedded JSON */
int gsvk_gsv_tensor_at(gsvk_gsv_t f, size_t i, gsvk_gsv_tensor* out);
int gsvk_gsv_find(gsvk_gsv_t f, const char* name, gsvk_gsv_tensor* out);
/* T2SEngine(const GsvFile&) (t2s_engine.cpp:544-630) on the device: the
 * dimensions from the embedded config (model_config.model hidden_dim, head,
 * linear_units, n_layer, vocab_size; embedding_dim == hidden_dim and EOS ==
 * vocab_size - 1 when present), the per-layer h.layers.<l>.* tensors,
 * ar_predict_layer.weight, ar_audio_embedding and ar_audio_position.alpha,
 * uploaded into a gsvk_t2s handle with `cap` KV slots.  The file may be
 * closed afterwards. */
int gsvk_t2s_create_from_gsv(gsvk_gsv_t f, int cap, gsvk_t2s_t* out);

/* ---- SoVITS latent path (sovits_engine.hpp:48-93 steps 1-5) ------------- */
/* codes -> RVQ decode (quantizer.hpp:26-38) -> nearest x2 -> TextEncoder
 * (enc_p.hpp: ssl_proj, relative-position encoders, text embedding, MRTE,
 * proj) -> m_p, logs_p -> z_p = m_p + noise * exp(logs_p) * noise_scale ->
 * reverse ResidualCouplingBlock (flow.hpp) -> z, the generator's input.
 * Convolutions run on the tensor cores with fp16 activations (the
 * reference's accelerated Conv1d path); attention is fp32. */
typedef struct gsvk_sovits_latent* gsvk_sovits_latent_t;
typedef struct {
  int ssl_dim;          /* 768 */
  int hidden;           /* 192; a multiple of 16, <= 512 */
  int filter;           /* 768 (FFN width) */
  int heads;            /* 2; hidden / heads a multiple of 32, <= 128 */
  int kernel;           /* 3 (FFN conv kernel, odd) */
  int window;           /* 4: relative tables of 2*window + 1 rows */
  int layers_ssl, layers_text, layers_2;   /* 3, 6, 3 */
  int mrte_hidden, mrte_heads;             /* 512, 4 */
  int gin;              /* 1024: speaker embedding width (flow condition) */
  int flows;            /* 4 coupling layers */
  int wn_layers;        /* 4 WaveNet layers per coupling layer */
  int wn_kernel;        /* 5 (odd) */
  float noise_scale;    /* 0.5 */
  size_t max_codes;     /* longest code sequence (frames = 2 x codes, <= 4096) */
  size_t max_phones;    /* longest phone sequence (<= 4096) */
} gsvk_sovits_latent_config;
/* Weights from named tensors with the .gsv names and shapes
 * (enc_p.*, flow.flows.*, quantizer.vq.layers.0._codebook.embed), read as
 * the reference's load_tensor_f16 / load_tensor_f32 do: a tensor's fp16 copy
 * when present, else its fp32 copy (rounded once for conv weights).  HOST
 * data; the codebook and text-embedding sizes come from the tensors.  A
 * missing or mis-sized tensor is GSVK_ERR_INVALID. */
int gsvk_sovits_latent_create(const gsvk_sovits_latent_config* cfg,
                              const gsvk_gsv_tensor* tensors, size_t n,
                              gsvk_sovits_latent_t* out);
/* The same from every tensor of an opened .gsv file. */
int gsvk_sovits_latent_create_from_gsv(gsvk_gsv_t f, const gsvk_sovits_latent_config* cfg,
                                       gsvk_sovits_latent_t* out);
int gsvk_sovits_latent_destroy(gsvk_sovits_latent_t h);
/* codes [n_codes], phones [n_phones]: HOST int64, checked against the
 * codebook / symbol table (GSVK_ERR_INVALID, as the reference throws).
 * ge [gin], ge_text [mrte_hidden], noise [hidden][2 n_codes] or NULL (no
 * noise: z_p = m_p): DEVICE fp32.  z, and m_p / logs_p unless NULL: DEVICE
 * fp32 [hidden][2 n_codes], channel-major like the reference's Tensor2D. */
int gsvk_sovits_latent_forward(gsvk_sovits_latent_t h, const int64_t* codes, size_t n_codes,
                               const int64_t* phones, size_t n_phones, const float* ge,
                               const float* ge_text, const float* noise, float* z, float* m_p,
                               float* logs_p, gsvk_stream_t stream);

/* ---- SV speaker encoder, ERes2NetV2 w24 s4 e4 (sv.cpp:130-885) ---------- */
/* fbank [frames][n_mels] -> embedding [C4 * F4] (C4 = 2048 channels, F4 =
 * n_mels after the three stride-2 stages): stem conv (fp32), 16 Res2Net
 * blocks, layer3_ds, fuse34 AFF, mean over time.  Convs are im2col + tensor
 * core GEMMs with fp16 operands (the reference's conv2d_f16); BatchNorm
 * runs in the reference's fp64 chain.  Weights by .gsv names (conv1.*,
 * bn1.*, layer{1..4}.{i}.*, layer3_ds.*, fuse34.*), HOST data. */
typedef struct gsvk_sv* gsvk_sv_t;
typedef struct {
  int n_mels;          /* 80 */
  size_t max_frames;   /* longest fbank a forward may take */
} gsvk_sv_config;
int gsvk_sv_create(const gsvk_sv_config* cfg, const gsvk_gsv_tensor* tensors, size_t n,
                   gsvk_sv_t* out);
int gsvk_sv_create_from_gsv(gsvk_gsv_t f, const gsvk_sv_config* cfg, gsvk_sv_t* out);
int gsvk_sv_destroy(gsvk_sv_t h);
size_t gsvk_sv_embedding_size(gsvk_sv_t h);
/* fbank: DEVICE fp32 [frames][n_mels]; emb: DEVICE fp32 [embedding_size]
 * (channel-major [C4][F4], SvEngine::emb_out). */
int gsvk_sv_forward(gsvk_sv_t h, const float* fbank, size_t frames, float* emb,
                    gsvk_stream_t stream);

/* ---- T2S autoregressive transformer: lifetime, generation, switches ----- */
int gsvk_t2s_destroy(gsvk_t2s_t h);
/* Copies a KV prefix (fp16 [L][src_rows][D] for K and V, host or device
 * memory) into slots [0, prefix) of every layer's cache. */
int gsvk_t2s_load_kv(gsvk_t2s_t h, const uint16_t* k_host, const uint16_t* v_host, size_t prefix,
                     size_t src_rows, gsvk_stream_t stream);
/* block_prefill (t2s_engine.cpp:881-1034) over all layers, in place on the
 * DEVICE rows x[S][D] (fp32), writing K/V into slots pos..pos+S-1.  Query q
 * sees slots below pos, the first text_len block slots and block slots <= q. */
int gsvk_t2s_prefill(gsvk_t2s_t h, float* x, size_t S, size_t pos, size_t text_len,
                     gsvk_stream_t stream);
/* generate (t2s_engine.cpp:1740-1900) over a cache whose slots [0, prefix)
 * are loaded: prompt prefill at prefix.., greedy decode with repetition
 * penalty 1.35 and the 11-step EOS mask.  stop_on_eos = 0 decodes through
 * EOS (fixed-length runs).  HOST prompt and outputs; synchronous.  margins
 * (optional, max_steps floats) receives top1 - top2 of each step's
 * penalised logits. */
int gsvk_t2s_generate(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_host, size_t P,
                      size_t max_steps, int stop_on_eos, int32_t* tokens_host,
                      float* margins_host, int* n_out, gsvk_stream_t stream);
/* The two halves of generate, DEVICE prompt, asynchronous on `stream`:
 * gsvk_t2s_prompt embeds the prompt (audio embedding + alpha * PE), runs the
 * prefill at slots prefix.. and computes the first logits;
 * gsvk_t2s_decode runs the whole greedy loop in one persistent kernel. */
int gsvk_t2s_prompt(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_dev, size_t P,
                    gsvk_stream_t stream);
int gsvk_t2s_decode(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_dev, size_t P,
                    size_t max_steps, int stop_on_eos, int32_t* tokens_dev, int* n_out_dev,
                    float* margins_dev, gsvk_stream_t stream);
/* Kernel launches one generate issues (prompt + decode). */
int gsvk_t2s_launches_per_generate(gsvk_t2s_t h);
/* Same as gsvk_t2s_generate with DEVICE prompt / outputs, asynchronous. */
int gsvk_t2s_generate_device(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_dev, size_t P,
                             size_t max_steps, int stop_on_eos, int32_t* tokens_dev,
                             int* n_out_dev, float* margins_dev, gsvk_stream_t stream);
/* Phase trace of the decode kernel (the reference's GSV_AR_TIMING probe,
 * t2s_engine.cpp:1906-1925, at phase granularity): when enabled, CTA 0
 * records the device clock (ns) at every phase boundary of the first 4 steps
 * of the next decode: per step 1040 slots, [0] step start, [1] sampled,
 * [2] logits done, [3] after the logits barrier, [16 + 16*l + 2*k] phase k of
 * layer l done, [.. + 1] its barrier passed, [16 + 16*l + 10..13] P1 after
 * LayerNorm, P1 after the weight wait, P4 after LayerNorm, P5 after the
 * activation load.  read_trace is synchronous. */
int gsvk_t2s_set_trace(gsvk_t2s_t h, int enable);
int gsvk_t2s_read_trace(gsvk_t2s_t h, unsigned long long* host_out, size_t n);
/* Which decode kernel gsvk_t2s_decode launches: 1 = persistent CTAs (one
 * per SM) with grid barriers (any shape), 2 = one 16-CTA
 * thread-block cluster with cluster barriers and distributed shared memory
 * (d_model 512, head_dim 32, ffn 2048, <= 16 heads, cap <= 4096, and a GPU
 * that places such a cluster), 3 = one thread-block cluster per attention
 * head with K/V tiles loaded by TMA, and vectors exchanged between clusters
 * through {value, epoch} words polled in global memory instead of grid
 * barriers (needs every cluster resident at once and its shared-memory plan
 * to fit; d_model, ffn and vocab up to 4096).  A kind the handle's shape or
 * GPU cannot run raises GSVK_ERR_UNSUPPORTED.  0 = the default: 3 where the
 * handle's shape and GPU can run it, 1 otherwise (the choice made at
 * gsvk_t2s_create).  All produce
 * identical tokens, margins, logits and KV.  gsvk_t2s_decode_kernel returns
 * the current choice (1, 2 or 3). */
int gsvk_t2s_set_decode_kernel(gsvk_t2s_t h, int kind);
int gsvk_t2s_decode_kernel(gsvk_t2s_t h);
/* Failure injection for tests (no counterpart in the reference): every
 * exchange poll of decode kernel 3 gives up after `polls` polls instead of
 * its own budget (seconds), records GSVK_ERR_TIMEOUT in the device status and
 * winds the launch down (no wait, every bulk copy drained before exit), so a
 * test can make a real device wait run out without faulting or hanging the
 * GPU.  0 restores the default.  Process-wide. */
int gsvk_set_spin_limit_for_test(uint32_t polls);
/* Check of the LayerNorm's reciprocal square root for tests (no counterpart
 * in the reference; the value it reproduces is kern.cpp:55's
 * (float)(1.0 / std::sqrt(v)) with correctly rounded double operations):
 * out[i] = the device routine every T2S LayerNorm uses, for n device doubles
 * v.  Synchronous on the stream. */
int gsvk_test_rstd(const double* v, float* out, size_t n, gsvk_stream_t stream);
/* Sampling of the decode steps: SamplingParams (t2s_engine.hpp:69-77) and
 * topk_sample (t2s_engine.cpp:1640-1737).  mode 0 (the default) is greedy;
 * mode 1 applies the repetition penalty rep_penalty once per distinct history
 * token, keeps the top_k logits (the reference's selection sort), divides by
 * temperature (<= 0: the best of the top k), takes a softmax (a fixed
 * Cody-Waite/Taylor exp in place of libm expf), cuts to the nucleus top_p
 * and draws from std::mt19937_64 seeded with seed for each generate call
 * (uniform = one 64-bit draw as float times 2^-64, as libc++'s
 * uniform_real_distribution<float> computes it).  seed 0 takes a seed from
 * the host clock (the reference uses std::random_device).  Top-k sampling
 * runs on decode kernel 3 only (GSVK_ERR_UNSUPPORTED otherwise).  Margins
 * stay top1 - top2 of the penalised logits.  NULL restores greedy. */
typedef struct {
  int mode;
  int top_k;
  float top_p;
  float temperature;
  float rep_penalty;
  unsigned long long seed;
} gsvk_t2s_sampling;
int gsvk_t2s_set_sampling(gsvk_t2s_t h, const gsvk_t2s_sampling* sp);
/* CTAs of the grid decode kernel (one per SM at most; 0 = every SM, the
 * default).  Results are identical for any count. */
int gsvk_t2s_set_decode_ctas(gsvk_t2s_t h, int ctas);
/* ---- batched T2S decode (config 3: concurrent utterances) -------------- */
/* B <= max_batch utterances decode together: every step streams the weights
 * once for all B tokens through tensor-core GEMMs (M = B), attends each
 * utterance over its own cache length and samples each greedily (penalty
 * 1.35 over its own history, 11-step EOS mask, no EOS stop).  fp16 GEMM
 * operands: parity with the batch-1 path is at GEMM tolerance.  Each
 * utterance has cfg->cap KV slots. */
typedef struct gsvk_t2s_batch* gsvk_t2s_batch_t;
int gsvk_t2s_batch_create(const gsvk_t2s_config* cfg, const gsvk_t2s_host_weights* w,
                          int max_batch, int max_steps, gsvk_t2s_batch_t* out);
int gsvk_t2s_batch_destroy(gsvk_t2s_batch_t h);
/* fp16 [L][src_rows][D] K/V (host or device memory) into slots [0, len) of
 * utterance b. */
int gsvk_t2s_batch_load_kv(gsvk_t2s_batch_t h, int b, const uint16_t* k_host,
                           const uint16_t* v_host, size_t len, size_t src_rows,
                           gsvk_stream_t stream);
/* HOST per-utterance cache lengths, PE origins, first input tokens and
 * histories ([B][n_hist], -1 ignored); resets the step counter. */
int gsvk_t2s_batch_begin(gsvk_t2s_batch_t h, int B, const int32_t* len, const int32_t* pe0,
                         const int32_t* first_tok, const int32_t* hist, int n_hist,
                         gsvk_stream_t stream);
/* Runs `steps` steps (asynchronous); use_graph captures one step as a CUDA
 * graph the first time and replays it. */
int gsvk_t2s_batch_run(gsvk_t2s_batch_t h, int steps, int use_graph, gsvk_stream_t stream);
/* HOST tokens / margins [steps][B] of the steps run since begin; synchronous. */
int gsvk_t2s_batch_read(gsvk_t2s_batch_t h, int steps, int32_t* tokens, float* margins);
int gsvk_t2s_batch_read_logits(gsvk_t2s_batch_t h, float* host_out);
int gsvk_t2s_batch_launches_per_step(gsvk_t2s_batch_t h);
/* Attention kernel of the batched step: 0 = one CTA per (utterance, 32-key
 * chunk), any supported d_model; 1 = persistent CTAs streaming 16-key chunks
 * of 128-key splits (d_model 256 / 512, the default there).  Both agree at
 * the batched path's GEMM tolerance.  Changing it drops the captured step
 * graph.  GSVK_ERR_UNSUPPORTED for a kernel the model cannot use. */
int gsvk_t2s_batch_set_attention(gsvk_t2s_batch_t h, int kind);
int gsvk_t2s_batch_attention(gsvk_t2s_batch_t h);

/* ---- T2S inspection (synchronous reads of the batch-1 engine) ----------- */
/* The logits the last step sampled from (raw, before the penalty); synchronous. */
int gsvk_t2s_read_logits(gsvk_t2s_t h, float* host_out);
/* The whole KV cache, fp16 [n_layers][cap][d_model] each (the layout of
 * gsvk_t2s_load_kv with src_rows = cap); synchronous. */
int gsvk_t2s_read_kv(gsvk_t2s_t h, uint16_t* k_host, uint16_t* v_host);

#ifdef __cplusplus
}
#endif
#endif
