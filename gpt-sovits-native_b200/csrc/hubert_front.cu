// hubert_front.cu — the HuBERT-base feature front-end on the device
// (GPT-SoVITS-native src/encoder/hubert.cpp:439-580): the 7-layer strided
// CNN feature extractor (GroupNorm on layer 0, GELU after every layer), the
// feature projection (LayerNorm, Linear), the grouped positional
// convolution (GELU, residual) and the encoder LayerNorm that feeds the
// transformer layers (gsvk_encoder_*).
//
// Activations are channels-last rows [T][C] fp32.  Each convolution is an
// im2col into fp16 rows (the reference also rounds the activations to fp16
// for its FMLAL / AMX GEMM, hubert.cpp:447-452) and one tensor-core GEMM
// C[T_out, C_out] = cols[T_out, Ci*k] . W[C_out, Ci*k]^T whose epilogue adds
// the bias, applies GELU and (positional conv) the residual.  The column
// order c*k + kk is the torch [out][in][k] weight order, so the weights are
// used as stored.  Layer 0 (Ci = 1, k = 10) pads its 10 columns to 16 with
// zeros (exact: the padded products are zero).
#include <cmath>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_hubert_front;

namespace gsvk {
namespace {

// cols[t][kk*ci + c] = f16(x[(t*stride + kk - pad) * x_ld + c]) for c < ci,
// kk < k, zero outside [0, t_in) and in the padding columns [ci*k, kp): tap-
// major columns, so that a tap's columns are one contiguous channels-last
// row of x (coalesced reads and writes); the weights are permuted to the same
// column order once at create.  One thread per (t, column).
__global__ void im2col_f16_kernel(const float* __restrict__ x, int x_ld, int t_in, int ci, int k,
                                  int stride, int pad, int t_out, int kp,
                                  uint16_t* __restrict__ cols) {
  const long long total = static_cast<long long>(t_out) * kp;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / kp);
    const int r = static_cast<int>(i - static_cast<long long>(t) * kp);
    uint16_t* row = cols + static_cast<size_t>(t) * kp;
    if (r < ci * k) {
      const int kk = r / ci, c = r - kk * ci;
      const int src = t * stride + kk - pad;
      const float v = (src >= 0 && src < t_in) ? x[static_cast<size_t>(src) * x_ld + c] : 0.f;
      row[r] = f2h(v);
    } else {
      row[r] = 0;
    }
  }
}

// GroupNorm with one group per channel (hubert.cpp:485-500): per channel the
// mean and the biased variance over T in fp64 (the reference's two passes),
// rstd = 1/sqrt(var + eps) in fp64, y = float((x - mu) * rstd * g + b), then
// GELU.  Three passes spread over the whole GPU: per (32-channel, row-chunk)
// block a partial sum (x, or (x - mu)^2 once mu is known) combined in a fixed
// order; per channel the chunk partials summed in chunk order; then the
// element-wise apply.
constexpr int kGnChunks = 64;

__global__ void __launch_bounds__(256) gn_partial_kernel(const float* __restrict__ y, int T, int C,
                                                         int rows, const double* __restrict__ mu,
                                                         double* __restrict__ part) {
  __shared__ double sp[8][33];
  const int cl = threadIdx.x & 31, rg = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  const int t0 = blockIdx.y * rows, t1 = min(T, t0 + rows);
  double s = 0.0;
  if (c < C) {
    const double m = mu ? mu[c] : 0.0;
    for (int t = t0 + rg; t < t1; t += 8) {
      const double v = static_cast<double>(y[static_cast<size_t>(t) * C + c]);
      s += mu ? (v - m) * (v - m) : v;
    }
  }
  sp[rg][cl] = s;
  __syncthreads();
  if (rg == 0 && c < C) {
    double a = 0.0;
    for (int r = 0; r < 8; ++r) a += sp[r][cl];
    part[static_cast<size_t>(blockIdx.y) * C + c] = a;
  }
}

// stat[c] = sum_r part[r][c] / T, then (rstd) 1 / sqrt(stat + eps).
__global__ void gn_stat_kernel(const double* __restrict__ part, int chunks, int T, int C,
                               double eps, int rstd, double* __restrict__ stat) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double a = 0.0;
  for (int r = 0; r < chunks; ++r) a += part[static_cast<size_t>(r) * C + c];
  a /= static_cast<double>(T);
  stat[c] = rstd ? 1.0 / sqrt(a + eps) : a;
}

__global__ void gn_apply_gelu_kernel(float* __restrict__ y, int T, int C,
                                     const double* __restrict__ mu,
                                     const double* __restrict__ rstd,
                                     const float* __restrict__ g, const float* __restrict__ b) {
  const long long n = static_cast<long long>(T) * C;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e % C);
    const double v = __dadd_rn(
        __dmul_rn(__dmul_rn(__dsub_rn(static_cast<double>(y[e]), mu[c]), rstd[c]),
                  static_cast<double>(g[c])),
        static_cast<double>(b[c]));
    y[e] = gelu_erf(static_cast<float>(v));
  }
}

}  // namespace
}  // namespace gsvk

using namespace gsvk;

struct gsvk_hubert_front {
  gsvk_hubert_front_config cfg{};
  int in_c[7] = {}, kp[7] = {};
  uint16_t* conv_w[7] = {};  // [conv_dim][kp] fp16 (layer 0 zero-padded to 16 columns)
  float *gn_g = nullptr, *gn_b = nullptr, *pln_g = nullptr, *pln_b = nullptr;
  uint16_t* proj_w = nullptr;
  float* proj_b = nullptr;
  uint16_t* pos_w = nullptr;  // fp16 [hidden][cg * pos_k]
  float *pos_b = nullptr, *eln_g = nullptr, *eln_b = nullptr;
  // workspaces for max_samples
  float *act0 = nullptr, *act1 = nullptr, *feat = nullptr, *pos_out = nullptr;
  uint16_t* cols = nullptr;
  uint16_t* feat16 = nullptr;
  double* gn_ws = nullptr;  // [kGnChunks][C] partials, then mu [C] and rstd [C]
  std::vector<void*> allocs;
};

namespace {

size_t conv_len(size_t t, int k, int s) { return t < static_cast<size_t>(k) ? 0 : (t - k) / s + 1; }

int dev_alloc(gsvk_hubert_front* h, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(GSVK_ERR_NOMEM, "hubert_front_create: %zu bytes", bytes);
  }
  h->allocs.push_back(*p);
  return GSVK_OK;
}

template <typename T>
int upload(gsvk_hubert_front* h, T** dst, const T* src, size_t n) {
  if (int rc = dev_alloc(h, reinterpret_cast<void**>(dst), n * sizeof(T))) return rc;
  return check_cuda(cudaMemcpy(*dst, src, n * sizeof(T), cudaMemcpyHostToDevice),
                    "hubert_front upload");
}

int run_gemm(const uint16_t* a, size_t lda, const uint16_t* b, size_t ldb, size_t M, size_t N,
             size_t K, const float* bias, const float* res, size_t ld_res, float* c, size_t ldc,
             int act, cudaStream_t st) {
  gsvk_gemm_args g{};
  g.a = a;
  g.lda = lda;
  g.b = b;
  g.ldb = ldb;
  g.M = M;
  g.N = N;
  g.K = K;
  g.bias = bias;
  g.residual = res;
  g.ld_res = ld_res;
  g.c = c;
  g.ldc = ldc;
  g.act = act;
  g.alpha = 1.f;
  return gemm_ex_run(&g, st, true);
}

unsigned grid_cap(long long n) {
  const long long cap = static_cast<long long>(sm_count()) * 8;
  long long b = (n + 255) / 256;
  return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

int launch_im2col(const float* x, int x_ld, int t_in, int ci, int k, int stride, int pad,
                  int t_out, int kp, uint16_t* cols, cudaStream_t st) {
  const long long total = static_cast<long long>(t_out) * kp;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  long long blocks = (total + 255) / 256;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  im2col_f16_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, x_ld, t_in, ci, k, stride, pad, t_out, kp,
                                                     cols);
  return check_launch("im2col_f16_kernel");
}

}  // namespace

extern "C" {

size_t gsvk_hubert_front_frames(gsvk_hubert_front_t h, size_t n) {
  if (!h) return 0;
  size_t t = n;
  for (int i = 0; i < 7; ++i) t = conv_len(t, h->cfg.conv_kernel[i], h->cfg.conv_stride[i]);
  return t;
}

int gsvk_hubert_front_destroy(gsvk_hubert_front_t h) {
  if (!h) return GSVK_OK;
  for (void* p : h->allocs) cudaFree(p);
  delete h;
  return GSVK_OK;
}

int gsvk_hubert_front_create(const gsvk_hubert_front_config* cfg,
                             const gsvk_hubert_front_weights* w, gsvk_hubert_front_t* out) {
  if (!cfg || !w || !out) return fail(GSVK_ERR_INVALID, "hubert_front_create: null argument");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  const int H = cfg->hidden, G = cfg->pos_groups, PK = cfg->pos_k;
  if (H <= 0 || G <= 0 || H % G || PK <= 0 || PK % 2 || cfg->max_samples == 0)
    return fail(GSVK_ERR_INVALID, "hubert_front_create: bad hidden / positional conv sizes");
  for (int i = 0; i < 7; ++i) {
    if (cfg->conv_dim[i] <= 0 || cfg->conv_dim[i] % 8 || cfg->conv_kernel[i] <= 0 ||
        cfg->conv_stride[i] <= 0 || !w->conv_w[i])
      return fail(GSVK_ERR_INVALID, "hubert_front_create: bad conv layer %d", i);
  }
  if ((H / G) * PK % 8 || H % 8 || !w->gn_g || !w->gn_b || !w->proj_ln_g || !w->proj_ln_b ||
      !w->proj_w || !w->proj_b || !w->pos_w || !w->pos_b || !w->enc_ln_g || !w->enc_ln_b)
    return fail(GSVK_ERR_INVALID, "hubert_front_create: null weight or unaligned group width");
  auto* h = new gsvk_hubert_front();
  h->cfg = *cfg;
  int rc = GSVK_OK;
  int ci = 1;
  size_t t = cfg->max_samples, max_cols = 0, max_act = 0;
  for (int i = 0; i < 7 && !rc; ++i) {
    const int k = cfg->conv_kernel[i], co = cfg->conv_dim[i];
    h->in_c[i] = ci;
    h->kp[i] = (ci * k + 15) / 16 * 16;
    t = conv_len(t, k, cfg->conv_stride[i]);
    if (t == 0) {
      rc = fail(GSVK_ERR_INVALID, "hubert_front_create: max_samples too short for the CNN");
      break;
    }
    max_cols = std::max(max_cols, t * h->kp[i]);
    max_act = std::max(max_act, t * static_cast<size_t>(co));
    // weights [co][ci][k] -> [co][kp] in the tap-major column order kk*ci + c
    // of the im2col (zero padding columns)
    std::vector<uint16_t> wp(static_cast<size_t>(co) * h->kp[i], 0);
    for (int o = 0; o < co; ++o)
      for (int c = 0; c < ci; ++c)
        for (int kk = 0; kk < k; ++kk)
          wp[static_cast<size_t>(o) * h->kp[i] + kk * ci + c] =
              w->conv_w[i][(static_cast<size_t>(o) * ci + c) * k + kk];
    rc = upload(h, &h->conv_w[i], wp.data(), wp.size());
    ci = co;
  }
  const int C6 = cfg->conv_dim[6], cg = H / G;
  const size_t T = t;  // frames at max_samples
  const size_t pos_cols = static_cast<size_t>(G) * T * cg * PK;
  if (!rc) rc = upload(h, &h->gn_g, w->gn_g, cfg->conv_dim[0]);
  if (!rc) rc = upload(h, &h->gn_b, w->gn_b, cfg->conv_dim[0]);
  if (!rc) rc = upload(h, &h->pln_g, w->proj_ln_g, C6);
  if (!rc) rc = upload(h, &h->pln_b, w->proj_ln_b, C6);
  if (!rc) rc = upload(h, &h->proj_w, w->proj_w, static_cast<size_t>(H) * C6);
  if (!rc) rc = upload(h, &h->proj_b, w->proj_b, H);
  if (!rc) {
    // the weight-normed fp32 positional weights, rounded to fp16 once
    // (hubert.cpp:538-539), [H][cg][PK] = group g's rows [g*cg, (g+1)*cg)
    // in the im2col's tap-major column order kk*cg + c
    std::vector<uint16_t> p16(static_cast<size_t>(H) * cg * PK);
    for (int o = 0; o < H; ++o)
      for (int c = 0; c < cg; ++c)
        for (int kk = 0; kk < PK; ++kk)
          p16[static_cast<size_t>(o) * cg * PK + kk * cg + c] = __half_as_ushort(
              __float2half_rn(w->pos_w[(static_cast<size_t>(o) * cg + c) * PK + kk]));
    rc = upload(h, &h->pos_w, p16.data(), p16.size());
  }
  if (!rc) rc = upload(h, &h->pos_b, w->pos_b, H);
  if (!rc) rc = upload(h, &h->eln_g, w->enc_ln_g, H);
  if (!rc) rc = upload(h, &h->eln_b, w->enc_ln_b, H);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->act0), max_act * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->act1), max_act * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->cols), std::max(max_cols, pos_cols) * 2);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->feat), T * H * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->pos_out), T * H * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->feat16), T * std::max(C6, H) * 2);
  if (!rc)
    rc = dev_alloc(h, reinterpret_cast<void**>(&h->gn_ws),
                   (static_cast<size_t>(kGnChunks) + 2) * cfg->conv_dim[0] * sizeof(double));
  if (rc) {
    gsvk_hubert_front_destroy(h);
    return rc;
  }
  *out = h;
  return GSVK_OK;
}

int gsvk_hubert_front_forward(gsvk_hubert_front_t h, const float* wav, size_t n, float* x,
                              gsvk_stream_t stream) {
  if (!h || !wav || !x) return fail(GSVK_ERR_INVALID, "hubert_front_forward: null argument");
  if (n > h->cfg.max_samples)
    return fail(GSVK_ERR_INVALID, "hubert_front_forward: %zu samples > max_samples %zu", n,
                h->cfg.max_samples);
  const size_t T = gsvk_hubert_front_frames(h, n);
  if (T == 0) return fail(GSVK_ERR_INVALID, "hubert_front_forward: too few samples");
  cudaStream_t st = as_cuda(stream);
  const gsvk_hubert_front_config& c = h->cfg;
  const float* in = wav;
  size_t t_in = n;
  float* bufs[2] = {h->act0, h->act1};
  int rc;
  for (int i = 0; i < 7; ++i) {
    const int k = c.conv_kernel[i], s = c.conv_stride[i], co = c.conv_dim[i], ci = h->in_c[i];
    const size_t t_out = conv_len(t_in, k, s);
    float* y = bufs[i & 1];
    if ((rc = launch_im2col(in, ci, (int)t_in, ci, k, s, 0, (int)t_out, h->kp[i], h->cols, st)))
      return rc;
    // conv (no bias); layer 0: GroupNorm then GELU, the others GELU in the epilogue
    if ((rc = run_gemm(h->cols, h->kp[i], h->conv_w[i], h->kp[i], t_out, co, h->kp[i], nullptr,
                       nullptr, 0, y, co, i == 0 ? GSVK_ACT_NONE : GSVK_ACT_GELU_ERF, st)))
      return rc;
    if (i == 0) {
      const int T = static_cast<int>(t_out);
      const int rows = (T + kGnChunks - 1) / kGnChunks, chunks = (T + rows - 1) / rows;
      double* part = h->gn_ws;
      double* mu = part + static_cast<size_t>(kGnChunks) * co;
      double* rstd = mu + co;
      const dim3 pg((co + 31) / 32, chunks);
      gn_partial_kernel<<<pg, 256, 0, st>>>(y, T, co, rows, nullptr, part);
      gn_stat_kernel<<<(co + 255) / 256, 256, 0, st>>>(part, chunks, T, co, 0.0, 0, mu);
      gn_partial_kernel<<<pg, 256, 0, st>>>(y, T, co, rows, mu, part);
      gn_stat_kernel<<<(co + 255) / 256, 256, 0, st>>>(part, chunks, T, co, (double)c.ln_eps, 1,
                                                        rstd);
      gn_apply_gelu_kernel<<<grid_cap(static_cast<long long>(T) * co), 256, 0, st>>>(
          y, T, co, mu, rstd, h->gn_g, h->gn_b);
      if ((rc = check_launch("group norm kernels"))) return rc;
    }
    in = y;
    t_in = t_out;
  }
  const int C6 = c.conv_dim[6], H = c.hidden, G = c.pos_groups, cg = H / G, PK = c.pos_k;
  float* cnn = const_cast<float*>(in);
  // feature projection: LayerNorm(C6) in place, fp16 activations, Linear + bias
  if ((rc = gsvk_layernorm_rows(cnn, h->pln_g, h->pln_b, cnn, T, C6, c.ln_eps, stream))) return rc;
  if ((rc = gsvk_f32_to_f16(cnn, h->feat16, T * C6, stream))) return rc;
  if ((rc = run_gemm(h->feat16, C6, h->proj_w, C6, T, H, C6, h->proj_b, nullptr, 0, h->feat, H,
                     GSVK_ACT_NONE, st)))
    return rc;
  // positional conv: per group, cols[g][t][kk*cg + j] = f16(feat[t + kk - PK/2][g*cg + j]);
  // out = GELU(conv + b) + feat (the first T of the T + 1 outputs: SamePad)
  for (int g = 0; g < G; ++g)  // group g's channels start at g*cg of a row of H
    if ((rc = launch_im2col(h->feat + g * cg, H, (int)T, cg, PK, 1, PK / 2, (int)T, cg * PK,
                            h->cols + static_cast<size_t>(g) * T * cg * PK, st)))
      return rc;
  std::vector<gsvk_gemm_args> grp(static_cast<size_t>(G));
  for (int g = 0; g < G; ++g) {
    gsvk_gemm_args& a = grp[g];
    a = gsvk_gemm_args{};
    a.a = h->cols + static_cast<size_t>(g) * T * cg * PK;
    a.lda = static_cast<size_t>(cg) * PK;
    a.b = h->pos_w + static_cast<size_t>(g) * cg * cg * PK;
    a.ldb = static_cast<size_t>(cg) * PK;
    a.M = T;
    a.N = cg;
    a.K = static_cast<size_t>(cg) * PK;
    a.bias = h->pos_b + g * cg;
    a.residual = h->feat + g * cg;
    a.ld_res = H;
    a.c = h->pos_out + g * cg;
    a.ldc = H;
    a.act = GSVK_ACT_GELU_ERF;
    a.alpha = 1.f;
  }
  if ((rc = gsvk_gemm_grouped_f16(grp.data(), grp.size(), stream))) return rc;
  // encoder.layer_norm
  return gsvk_layernorm_rows(h->pos_out, h->eln_g, h->eln_b, x, T, H, c.ln_eps, stream);
}

}  // extern "C"
