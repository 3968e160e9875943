/* oracle.h — CPU restatement of the GPT-SoVITS-native `src/kern` GEMM/GEMV
 * family and of the callers on its hot path (T2S decode, SoVITS conv stack).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path and the timed CPU baseline; product code never links or calls it.
 *
 * Every function cites the reference file:line whose arithmetic it restates
 * (paths relative to the reference project root).  fp16 values travel as
 * IEEE binary16 bit patterns in uint16_t, exactly as in the reference.
 *
 * Parity is pinned against the reference's own golden vectors
 * (tests/kern_golden, exported by tools/export_kern_golden.py) and against
 * torch CPU for the operators those vectors do not cover.
 */
#ifndef GSV_ORACLE_H
#define GSV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Thread pool used for the row-band partitions (gemv.cpp:117-126,
 * gemv_fmlal.cpp:195-204).  n <= 1 runs everything on the caller thread. */
void ora_set_threads(int n);
int ora_get_threads(void);

/* ---- fp16 conversion -------------------------------------------------- */
/* gemv_fmlal.cpp:23-35: round-to-nearest-even fp32 -> fp16 bits. */
void ora_f32_to_f16(const float* src, uint16_t* dst, size_t n);
/* accel.cpp:10-22: exact widening fp16 -> fp32. */
void ora_f16_to_f32(const uint16_t* src, float* dst, size_t n);

/* ---- GEMV / GEMM ------------------------------------------------------ */
/* gemv.cpp:21-32  y[o] = sum_k f32(W[o,k]) * x[k], sequential fp32. */
void ora_gemv_f16w_f32acc_ref(const uint16_t* w, const float* x, float* y,
                              size_t out, size_t in);
/* gemv.cpp:36-126  4-row blocked, two 4-lane accumulators per row. */
void ora_gemv_f16w_f32acc(const uint16_t* w, const float* x, float* y,
                          size_t out, size_t in);
/* gemv_fmlal.cpp:40-130  fp16 x, 8 x 4-lane accumulators, 64-wide steps. */
void ora_gemv_f16x_fmlal(const uint16_t* w, const uint16_t* xh, float* y,
                         size_t out, size_t in);
/* gemv_fmlal.cpp:140-204  C[M,N] = A[M,K] * B[N,K]^T, fp16 in, fp32 acc. */
void ora_gemm_f16x_fmlal(const uint16_t* a, const uint16_t* b, float* c,
                         size_t M, size_t N, size_t K);
/* accel.hpp:22-30 / accel.cpp:25-33  row-major cblas_sgemm semantics;
 * beta == 0 never reads C. */
void ora_sgemm(char transa, char transb, int M, int N, int K, float alpha,
               const float* A, int lda, const float* B, int ldb, float beta,
               float* C, int ldc);

/* Epilogue codes shared with the CUDA library. */
enum {
  ORA_ACT_NONE = 0,
  ORA_ACT_RELU = 1,
  ORA_ACT_GELU_ERF = 2,
  ORA_ACT_LEAKY = 3
};

/* bert_ops.hpp:225-258 / accel.hpp:70-78 (DenseF16 view path):
 * y[T,out] = act( f16(x)[T,in] . W[out,in]^T + b ).  bias may be NULL. */
void ora_linear_f16(const float* x, size_t T, size_t in, const uint16_t* w,
                    size_t out, const float* bias, int act, float slope,
                    float* y);

/* ---- support primitives (kern.cpp, bert_ops.hpp, nn_ops.hpp) ----------- */
void ora_layernorm(const float* x, const float* g, const float* b, float* y,
                   size_t n, double eps);                     /* kern.cpp:27 */
void ora_rmsnorm(const float* x, const float* g, float* y, size_t n,
                 double eps);                                 /* kern.cpp:11 */
void ora_softmax(const float* x, float* y, size_t n);         /* kern.cpp:62 */
void ora_relu(const float* x, float* y, size_t n);            /* kern.cpp:85 */
void ora_silu(const float* x, float* y, size_t n);            /* kern.cpp:79 */
void ora_gelu_erf(const float* x, float* y, size_t n);   /* bert_ops.hpp:25 */
void ora_leaky_relu(const float* x, float* y, size_t n,
                    float slope);                         /* nn_ops.hpp:48 */

/* ---- SoVITS convolutions ---------------------------------------------- */
/* conv1d.hpp:109-194  same-padding dilated Conv1d on channel-major
 * x[Ci,T] -> y[Co,T].  w is the torch layout [Co,Ci,k] in fp16 bits;
 * bias may be NULL.  round_in != 0 rounds the activations to fp16 before the
 * GEMM (the accelerated path's im2col_to_panel_f16, sovits_types.hpp:178);
 * round_in == 0 is the fp32 sgemm path. */
void ora_conv1d(const float* x, size_t Ci, size_t T, const uint16_t* w,
                const float* bias, size_t Co, size_t k, size_t dil,
                int round_in, float* y);
/* conv1d.hpp:250-359  ConvTranspose1d(k, stride u, pad (k-u)/2):
 * x[Ci,T] -> y[Co,T*u].  w is the torch layout [Ci,Co,k]. */
void ora_convt1d(const float* x, size_t Ci, size_t T, const uint16_t* w,
                 const float* bias, size_t Co, size_t k, size_t u,
                 int round_in, float* y);

/* dec.hpp:265-345  HiFi-GAN generator (ResBlock1 variant) without the cond
 * term.  Weight order in w/b (n_stages = 5, 3 resblocks, 3 pairs):
 *   [0] conv_pre;  then per stage s: [1 + s*19] ups[s];
 *   [1 + s*19 + 1 + j*6 + p*2 + 0] resblock j convs1[p],
 *   [1 + s*19 + 1 + j*6 + p*2 + 1] resblock j convs2[p];
 *   [1 + 5*19] conv_post (bias may be NULL).
 * ch0 = conv_pre output channels; channel count halves per stage. */
typedef struct {
  int n_stages;
  int in_ch;            /* latent channels (192) */
  int ch0;              /* conv_pre output channels */
  int conv_pre_k;       /* 7 */
  int conv_post_k;      /* 7 */
  int up_rate[8];
  int up_k[8];
  int res_k[3];         /* {3, 7, 11} */
  int res_dil[3];       /* {1, 3, 5} */
  float lrelu_slope;    /* 0.1 */
  float post_slope;     /* 0.01 */
} ora_decoder_cfg;

size_t ora_decoder_out_len(const ora_decoder_cfg* cfg, size_t T);
void ora_decoder_forward(const ora_decoder_cfg* cfg,
                         const uint16_t* const* w, const float* const* b,
                         const float* z, size_t T, int round_in, float* wav);

/* ---- T2S autoregressive transformer ------------------------------------ */
typedef struct {
  int n_layers, d_model, n_heads, ffn, vocab;
  float ln_eps;
  float alpha_audio;
} ora_t2s_dims;

typedef struct {
  const uint16_t* wqkv; const float* bqkv;  /* [L][3D][D], [L][3D] */
  const uint16_t* wout; const float* bout;  /* [L][D][D],  [L][D]  */
  const uint16_t* w1;   const float* b1;    /* [L][F][D],  [L][F]  */
  const uint16_t* w2;   const float* b2;    /* [L][D][F],  [L][D]  */
  const float* n1g; const float* n1b;       /* [L][D] */
  const float* n2g; const float* n2b;       /* [L][D] */
  const uint16_t* wpred;                    /* [V][D], no bias */
  const uint16_t* audio_emb;                /* [V][D] */
} ora_t2s_weights;

/* t2s_engine.cpp:711-720  sinusoidal position row, fp32 expressions. */
void ora_t2s_pe_row(int d_model, size_t pos, float* pe);

/* T2S numerics.  The reference leaves the association of its sums to NEON
 * register blocking and Accelerate; this oracle fixes ONE canonical order that
 * the device kernels reproduce bit for bit:
 *   - every dot product: the gemv_fmlal.cpp:40-109 order (8 x 4 accumulators
 *     over 64-element steps, low then high half, vaddv per group, groups summed
 *     in order), for fp16 and fp32 activations alike;
 *   - LayerNorm: kern.cpp:27-58 (8-lane fp32 sums, fp64 combine);
 *   - attention scores: dot_f16kv (t2s_engine.cpp:69-99);
 *   - softmax: chunks of 64 slots (sequential sums inside a chunk, chunk
 *     weights exp(m_c - M)) with a deterministic Cody-Waite/Taylor exp within
 *     2 ulp of expf.
 * Rounding points are the reference's: fp16(x) before QKV, out-proj and W1
 * (GEMV16), fp16 K/V storage (KV16), fp32 activations into W2 and the logits.
 *
 * t2s_engine.cpp:1036-1119 with KV16 && GEMV16 (the `--fp16-all` mode):
 * one post-LN decode layer over x[D] in place; appends k/v at slot pos into
 * kcache/vcache (token-major [cap][D] fp16) and attends over [0, pos]. */
void ora_t2s_decode_layer(const ora_t2s_dims* d, const ora_t2s_weights* w,
                          int layer, float* x, size_t pos, uint16_t* kcache,
                          uint16_t* vcache);

/* The same layer written line by line as t2s_engine.cpp:1036-1119 (KV16 &&
 * GEMV16) where the canonical order above departs from it: attention takes
 * kern::softmax over all len slots (kern.cpp:62-73: sequential max, libm
 * expf, sequential sum, multiply by 1/sum) and accumulates normalised p * v
 * slot by slot (accum_f16kv); W2 is the resident fp32 DenseF16 (accel.hpp:
 * 85-92), i.e. sgemm at M = 1, restated as one FMA chain per row (ora_sgemm's
 * order: Accelerate's blocking is closed).  QKV, out-proj, W1 (gemv_fmlal),
 * the scores (dot_f16kv) and LayerNorm are the same in both. */
void ora_t2s_decode_layer_literal(const ora_t2s_dims* d, const ora_t2s_weights* w,
                                  int layer, float* x, size_t pos, uint16_t* kcache,
                                  uint16_t* vcache);

/* t2s_engine.cpp:881-1034 with KV16: S rows x[S][D] at absolute slots
 * pos..pos+S-1.  Query q sees every slot below pos, the first text_len
 * slots of the block, and block slots <= q (pos == 0 reproduces the
 * reference's text-prefix mask exactly).  All four projections take
 * fp16-rounded activations (the DenseF16 view / accelerated-panel semantics,
 * accel.hpp:70-78). */
void ora_t2s_prefill_layer(const ora_t2s_dims* d, const ora_t2s_weights* w,
                           int layer, float* x, size_t S, size_t pos,
                           size_t text_len, uint16_t* kcache,
                           uint16_t* vcache);

/* t2s_engine.cpp:1062-1087  one query per head over slots [0, len) of a
 * token-major fp16 cache (rows of row_stride halves, head h at column
 * h*head_dim), canonical chunked softmax; out [n_heads*head_dim]. */
void ora_attention_decode(const float* q, const uint16_t* kc, const uint16_t* vc, size_t len,
                          size_t n_heads, size_t head_dim, size_t row_stride, float scale,
                          float* out);

/* t2s_engine.cpp:1594-1636  repetition penalty 1.35 once per distinct
 * history token, EOS column excluded while !eos_allowed, argmax. */
int ora_t2s_greedy_sample(float* logits, int vocab, const int32_t* history,
                          size_t n_hist, int eos_allowed, int* raw_argmax);

/* t2s_engine.cpp:1740-1900  prompt prefill at slots prefix..prefix+P-1 over
 * a caller-provided fp16 KV prefix, then greedy decode.  kcache/vcache are
 * [L][cap][D] fp16 with the first `prefix` slots filled by the caller;
 * cap >= prefix + P + max_steps.  stop_on_eos = 0 keeps decoding through
 * EOS (fixed-length benchmark runs).  Returns the number of sampled tokens
 * written to tokens_out; margins_out (optional) receives per-step
 * top1 - top2 of the penalised logits; last_logits (optional, vocab floats)
 * the raw logits the final step sampled from. */
int ora_t2s_generate(const ora_t2s_dims* d, const ora_t2s_weights* w,
                     uint16_t* kcache, uint16_t* vcache, size_t cap,
                     size_t prefix, const int32_t* prompt, size_t P,
                     size_t max_steps, int stop_on_eos, int32_t* tokens_out,
                     float* margins_out, float* last_logits);

/* ora_t2s_generate with the decode layers and logits head selectable:
 * literal = 0 is ora_t2s_generate; literal != 0 decodes through
 * ora_t2s_decode_layer_literal and takes the logits through the fp32 DenseF16
 * order (predict_layer_fp, t2s_engine.cpp:704-708).  The prompt prefill is
 * the canonical one in both.  all_logits (optional, max_steps x vocab)
 * receives the raw logits every step sampled from. */
int ora_t2s_generate_ex(const ora_t2s_dims* d, const ora_t2s_weights* w,
                        uint16_t* kcache, uint16_t* vcache, size_t cap,
                        size_t prefix, const int32_t* prompt, size_t P,
                        size_t max_steps, int stop_on_eos, int literal,
                        int32_t* tokens_out, float* margins_out, float* all_logits);

/* SamplingParams (t2s_engine.hpp:69-77): mode 0 greedy, 1 top-k. */
typedef struct {
  int mode;
  int top_k;
  float top_p;
  float temperature;
  float rep_penalty;
  unsigned long long seed;
} ora_sampling;

/* ora_t2s_generate with sampling params: mode 1 samples every step with
 * topk_sample (t2s_engine.cpp:1640-1737) from a std::mt19937_64 seeded with
 * sp->seed (t2s_engine.cpp:1814-1818); margins_out receives top1 - top2 of
 * the penalised logits. */
int ora_t2s_generate_sampled(const ora_t2s_dims* d, const ora_t2s_weights* w,
                             uint16_t* kcache, uint16_t* vcache, size_t cap,
                             size_t prefix, const int32_t* prompt, size_t P,
                             size_t max_steps, int stop_on_eos, const ora_sampling* sp,
                             int32_t* tokens_out, float* margins_out);

/* ---- HuBERT feature front-end (hubert.cpp:476-580) ----------------------- */
typedef struct {
  int conv_dim[7], conv_kernel[7], conv_stride[7];
  int hidden, pos_k, pos_groups;
  double ln_eps;
} ora_hubert_front_cfg;
typedef struct {
  const uint16_t* conv_w[7];      /* fp16 [conv_dim][in][k] */
  const float* gn_g; const float* gn_b;
  const float* proj_ln_g; const float* proj_ln_b;
  const uint16_t* proj_w; const float* proj_b;
  const float* pos_w; const float* pos_b;   /* fp32 [hidden][hidden/groups][pos_k] */
  const float* enc_ln_g; const float* enc_ln_b;
} ora_hubert_front_weights;
/* Frames of n samples. */
size_t ora_hubert_front_frames(const ora_hubert_front_cfg* c, size_t n);
/* The CNN stack (im2col rounded to fp16, gemm_f16x_fmlal, GroupNorm in fp64
 * on layer 0, GELU), the feature projection (LayerNorm, DenseF16 view +
 * bias), the grouped positional conv (fp16-rounded weights, + bias, GELU,
 * SamePad, residual) and the encoder LayerNorm: out [frames][hidden]. */
void ora_hubert_front(const ora_hubert_front_cfg* c, const ora_hubert_front_weights* w,
                      const float* wav, size_t n, float* out);

/* ---- SoVITS latent path (sovits_engine.hpp:48-93 steps 1-5) ------------ */
/* Named tensors, the .gsv names and layouts (sovits_types.hpp:38-95): a
 * tensor offers an fp16 copy, an fp32 copy or both. */
typedef struct {
  const char* name;
  const float* f32;
  const uint16_t* f16;
  uint64_t numel;
} ora_named;
typedef struct {
  int ssl_dim;          /* 768 */
  int hidden;           /* 192 */
  int filter;           /* 768 */
  int heads;            /* 2 */
  int kernel;           /* 3 */
  int window;           /* 4 (relative tables of 2W+1 rows) */
  int layers_ssl, layers_text, layers_2;   /* 3, 6, 3 */
  int mrte_hidden, mrte_heads;             /* 512, 4 */
  int gin;              /* 1024 */
  int flows;            /* 4 */
  int wn_layers;        /* 4 */
  int wn_kernel;        /* 5 */
  float noise_scale;    /* 0.5 */
} ora_sovits_latent_cfg;
/* codes[Tc] -> RVQ decode, nearest x2, TextEncoder (ssl_proj, rel-MHA
 * encoders, text embedding, MRTE, proj) -> m_p, logs_p [hidden][2Tc];
 * z_p = m_p + noise * exp(logs_p) * noise_scale (noise [hidden][2Tc] or
 * NULL); reverse flow (4 x flip + mean-only coupling with a WaveNet) -> z.
 * Conv1d inputs are rounded to fp16 (the accelerated path); the cond layer
 * (one frame) stays fp32.  Returns 0, -1 for a missing / mis-sized tensor,
 * -2 for a code or phone id out of range. */
int ora_sovits_latent(const ora_sovits_latent_cfg* c, const ora_named* t, size_t n,
                      const int64_t* codes, size_t Tc, const int64_t* phones, size_t Tt,
                      const float* ge, const float* ge_text, const float* noise,
                      float* m_p, float* logs_p, float* z);

/* ---- SV speaker encoder, ERes2NetV2 w24 s4 e4 (sv.cpp:130-885) --------- */
/* fbank [frames][n_mels] -> embedding [C4 * n_mels / 8] (C4 = 2048): the
 * fp32 stem conv (sgemm), four Res2Net stages (conv2d_f16: im2col rounded
 * to fp16, gemm_f16x_fmlal), BatchNorm in the fp64 chain, relu20, AFF
 * fusions, layer3_ds, fuse34 and the mean over time.  Named tensors as in
 * the .gsv.  Returns the embedding size, 0 for a missing tensor. */
size_t ora_sv_forward(const ora_named* t, size_t n, const float* fbank, size_t frames,
                      int n_mels, float* emb);
/* conv2d_f16 (sv.cpp:196-258) on its own: in [c_in][h][w] fp32, w16
 * [c_out][c_in*kh*kw] -> out [c_out][oh*ow]. */
void ora_sv_conv2d_f16(const float* in, int c_in, int h, int w, const uint16_t* w16, int c_out,
                       int kh, int kw, int stride, int pad, float* out);

/* ---- encoders (BERT / HuBERT post-LN layer) ---------------------------- */
typedef struct {
  int layers, hidden, heads, ffn;
  double eps;  /* 1e-12 RoBERTa, 1e-5 HuBERT */
} ora_encoder_dims;

typedef struct {
  const uint16_t* wqkv; const float* bqkv; /* [L][3C][C] (q, k, v rows), [L][3C] */
  const uint16_t* wo;   const float* bo;   /* [L][C][C], [L][C] */
  const float* ln1g; const float* ln1b;    /* [L][C] */
  const uint16_t* wi;   const float* bi;   /* [L][F][C], [L][F] */
  const uint16_t* wf;   const float* bf;   /* [L][C][F], [L][C] */
  const float* ln2g; const float* ln2b;    /* [L][C] */
} ora_encoder_weights;

/* bert_ops.hpp:347-400 (see oracle.cpp): one layer over x [B*T][C] in place;
 * valid (optional, B ints) masks keys >= valid[b]. */
void ora_encoder_layer(const ora_encoder_dims* d, const ora_encoder_weights* w, int layer,
                       float* x, int B, int T, const int* valid);

#ifdef __cplusplus
}
#endif
#endif
