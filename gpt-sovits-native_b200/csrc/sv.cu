// sv.cu — the SV speaker encoder (ERes2NetV2 w24 s4 e4) on the device
// (GPT-SoVITS-native src/encoder/sv.cpp:130-885, the default path): the
// fp32 stem conv, four Res2Net stages (1x1 / 3x3 / strided convs, BatchNorm
// in the fp64 chain, relu20, hierarchical splits with AFF fusion in stages
// 3-4), layer3_ds, the fuse34 AFF and the mean over time.
//
// Activations stay channel-major [C][H][W] fp32 as in the reference.  A
// convolution is an im2col into fp16 rows cols[S][K] (K = c_in*kh*kw in the
// torch weight order, so weights are used as stored) and one tensor-core
// GEMM out[c_out][S] = W[c_out][K] . cols[S][K]^T (fp32 accumulate), the
// arithmetic of the reference's conv2d_f16 (im2col rounded to fp16,
// gemm_f16x_fmlal).  1x1 stride-1 convs skip the gather: their cols are the
// fp16 transpose of the input.  The stem conv (c_in = 1, K = 9) keeps fp32
// operands through the sgemm kernel, as the reference's conv2d does.
#include <algorithm>
#include <cmath>
#include <map>
#include <string>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_sv;

namespace gsvk {
namespace {

constexpr int kActRelu = 1, kActRelu20 = 2, kActSilu = 3;  // 0: identity

__device__ __forceinline__ float relu20(float v) { return v < 0.f ? 0.f : (v > 20.f ? 20.f : v); }

// Bn::apply (sv.cpp:132-145): float((double(x) - mu) * a + beta), each
// double operation rounded separately.
__device__ __forceinline__ float bn64(float x, double a, double mu, double beta) {
  return static_cast<float>(__dadd_rn(__dmul_rn(__dsub_rn(static_cast<double>(x), mu), a), beta));
}

__device__ __forceinline__ float act_apply(float v, int act) {
  if (act == kActRelu) return v < 0.f ? 0.f : v;
  if (act == kActRelu20) return relu20(v);
  if (act == kActSilu) return __fdiv_rn(v, __fadd_rn(1.f, expf(-v)));  // kern.cpp:80-83
  return v;
}

// cols[s][k] = x[c][oy*stride - pad + ky][ox*stride - pad + kx], k = (c*kh +
// ky)*kw + kx, zero outside the image.  One thread per (s, c): consecutive
// threads take consecutive output pixels (coalesced reads of a row).
template <typename TO>
__global__ void im2col2d_kernel(const float* __restrict__ x, int c_in, int h, int w, int kh,
                                int kw, int stride, int pad, int ow, int S, TO* __restrict__ cols) {
  const long long n = static_cast<long long>(S) * c_in;
  const int K = c_in * kh * kw;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e / S), s = static_cast<int>(e - static_cast<long long>(c) * S);
    const int oy = s / ow, ox = s - oy * ow;
    const float* plane = x + static_cast<size_t>(c) * h * w;
    TO* dst = cols + static_cast<size_t>(s) * K + static_cast<size_t>(c) * kh * kw;
    for (int ky = 0; ky < kh; ++ky) {
      const int iy = oy * stride - pad + ky;
      for (int kx = 0; kx < kw; ++kx) {
        const int ix = ox * stride - pad + kx;
        const float v =
            (iy >= 0 && iy < h && ix >= 0 && ix < w) ? plane[static_cast<size_t>(iy) * w + ix] : 0.f;
        if constexpr (sizeof(TO) == 2)
          dst[ky * kw + kx] = f2h(v);
        else
          dst[ky * kw + kx] = v;
      }
    }
  }
}

// out[s][c] = fp16(c < ca ? a[c][s] : b[c - ca][s]) through 32 x 32 shared
// tiles (the transposes of 1x1 convs and of the AFF concatenation,
// f32_trans_to_f16).
__global__ void __launch_bounds__(256) transpose_f16_kernel(const float* __restrict__ a,
                                                            const float* __restrict__ b, int ca,
                                                            int C, int S,
                                                            uint16_t* __restrict__ out) {
  __shared__ float tile[32][33];
  const int s0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8) {
    const int c = c0 + r, s = s0 + tx;
    float v = 0.f;
    if (c < C && s < S)
      v = c < ca ? a[static_cast<size_t>(c) * S + s] : b[static_cast<size_t>(c - ca) * S + s];
    tile[r][tx] = v;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int s = s0 + r, c = c0 + tx;
    if (s < S && c < C) out[static_cast<size_t>(s) * C + c] = f2h(tile[tx][r]);
  }
}

// [T][F] -> [F][T] (the fbank as a one-channel F x T image, sv.cpp:805-809).
__global__ void fbank_to_image_kernel(const float* __restrict__ fb, int T, int F,
                                      float* __restrict__ img) {
  const long long n = static_cast<long long>(T) * F;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int f = static_cast<int>(e / T), t = static_cast<int>(e - static_cast<long long>(f) * T);
    img[e] = fb[static_cast<size_t>(t) * F + f];
  }
}

// y = act(BN(x + bias)) per channel of [C][S] (bias optional: the AFF
// convs' per-channel bias, added as its own fp32 rounding like the
// reference's row loop); y2 (optional) gets a copy.
__global__ void bn_act_kernel(const float* x, const float* __restrict__ bias, int C, int S,
                              const double* __restrict__ bn, int act, float* y,
                              float* __restrict__ y2) {
  const long long n = static_cast<long long>(C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e / S);
    const float u = bias ? __fadd_rn(x[e], bias[c]) : x[e];
    const float v = act_apply(bn64(u, bn[3 * c], bn[3 * c + 1], bn[3 * c + 2]), act);
    y[e] = v;
    if (y2) y2[e] = v;
  }
}

// Block tail (sv.cpp:612-643): out = relu20(BN3(a) + (sc_bn ? BNsc(b) : b)).
__global__ void block_tail_kernel(const float* a, const double* __restrict__ bn3,
                                  const float* __restrict__ b, const double* __restrict__ bnsc,
                                  int C, int S, float* out) {
  const long long n = static_cast<long long>(C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e / S);
    const float u = bn64(a[e], bn3[3 * c], bn3[3 * c + 1], bn3[3 * c + 2]);
    const float r = bnsc ? bn64(b[e], bnsc[3 * c], bnsc[3 * c + 1], bnsc[3 * c + 2]) : b[e];
    out[e] = relu20(__fadd_rn(u, r));
  }
}

// AFF output (sv.cpp:506-520): t = tanh(BN2(at + b2)); out = x (1 + t) +
// ds (1 - t).
__global__ void aff_combine_kernel(const float* __restrict__ at, const float* __restrict__ b2,
                                   const double* __restrict__ bn, const float* x,
                                   const float* __restrict__ ds, int C, int S, float* out) {
  const long long n = static_cast<long long>(C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e / S);
    const float u = __fadd_rn(at[e], b2[c]);
    const float t = tanhf(bn64(u, bn[3 * c], bn[3 * c + 1], bn[3 * c + 2]));
    out[e] = __fadd_rn(__fmul_rn(x[e], __fadd_rn(1.f, t)), __fmul_rn(ds[e], __fsub_rn(1.f, t)));
  }
}

__global__ void add_inplace_kernel(float* __restrict__ y, const float* __restrict__ x,
                                   long long n) {
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x)
    y[e] = __fadd_rn(y[e], x[e]);
}

// emb[r] = float(sum_t double(x[r][t]) / w) for the rows r = (c, fy)
// (sv.cpp:870-879); one warp per row.
__global__ void mean_rows_kernel(const float* __restrict__ x, int rows, int w,
                                 float* __restrict__ emb) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  double acc = 0.0;
  for (int t = lane; t < w; t += 32) acc += static_cast<double>(x[static_cast<size_t>(r) * w + t]);
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) emb[r] = static_cast<float>(acc / w);
}

unsigned grid_for(long long n) {
  const long long cap = static_cast<long long>(sm_count()) * 8;
  long long b = (n + 255) / 256;
  return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace gsvk

using namespace gsvk;

namespace {

struct SvConv {
  uint16_t* w = nullptr;  // [c_out][c_in*kh*kw]
  int co = 0, ci = 0, k = 1;
};

struct SvAffD {
  SvConv w1, w2;
  float *b1 = nullptr, *b2 = nullptr;
  double *bn1 = nullptr, *bn2 = nullptr;  // (a, mu, beta) per channel
  int inter = 0, ch = 0;
};

struct SvBlockD {
  bool aff = false, has_sc = false;
  int width = 0, scale = 4, exp = 0, stride = 1, c_in = 0;
  SvConv conv1, conv3, sc;
  std::vector<SvConv> convs;
  double *bn1 = nullptr, *bn3 = nullptr, *sc_bn = nullptr;
  std::vector<double*> bns;
  std::vector<SvAffD> fuses;
};

}  // namespace

struct gsvk_sv {
  gsvk_sv_config cfg{};
  std::vector<void*> allocs;
  float* stem_w = nullptr;  // fp32 [m_ch][9]
  double* stem_bn = nullptr;
  int m_ch = 0;
  std::vector<SvBlockD> blocks[4];
  SvConv l3ds;
  SvAffD fuse34;
  int c3 = 0, c4 = 0;
  // workspaces
  float *img = nullptr, *A = nullptr, *B = nullptr, *c1 = nullptr, *tmp2 = nullptr, *sp = nullptr;
  float *sc = nullptr, *ds = nullptr, *att = nullptr, *at = nullptr, *cols32 = nullptr;
  uint16_t* cols = nullptr;
};

namespace {

using TensorMap = std::map<std::string, const gsvk_gsv_tensor*>;

const gsvk_gsv_tensor* find(const TensorMap& m, const std::string& n) {
  auto it = m.find(n);
  return it == m.end() || (!it->second->f32 && !it->second->f16) ? nullptr : it->second;
}

int missing(const std::string& n) {
  return fail(GSVK_ERR_INVALID, "sv_create: missing tensor %s", n.c_str());
}

int dev_alloc(gsvk_sv* h, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
    cudaGetLastError();
    return fail(GSVK_ERR_NOMEM, "sv_create: %zu bytes", bytes);
  }
  h->allocs.push_back(*p);
  return GSVK_OK;
}

template <typename T>
int upload(gsvk_sv* h, T** dst, const std::vector<T>& src) {
  if (int rc = dev_alloc(h, reinterpret_cast<void**>(dst), src.size() * sizeof(T))) return rc;
  return check_cuda(cudaMemcpy(*dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice),
                    "sv upload");
}

// vec_any (sv.cpp:74-84).
int vec_any(const TensorMap& m, const std::string& n, std::vector<float>* v) {
  const gsvk_gsv_tensor* t = find(m, n);
  if (!t) return missing(n);
  v->resize(t->numel);
  for (size_t i = 0; i < v->size(); ++i)
    (*v)[i] = t->f16 ? __half2float(__ushort_as_half(t->f16[i])) : t->f32[i];
  return GSVK_OK;
}

// load_bn + the per-channel (a = g / sqrt(var + 1e-5), mu, beta) of the
// fp64 chain (sv.cpp:132-145), computed once.
int load_bn(gsvk_sv* h, const TensorMap& m, const std::string& p, int c, double** out) {
  std::vector<float> g, b, mu, var;
  int rc = vec_any(m, p + ".weight", &g);
  if (!rc) rc = vec_any(m, p + ".bias", &b);
  if (!rc) rc = vec_any(m, p + ".running_mean", &mu);
  if (!rc) rc = vec_any(m, p + ".running_var", &var);
  if (rc) return rc;
  if (static_cast<int>(g.size()) != c || b.size() != g.size() || mu.size() != g.size() ||
      var.size() != g.size())
    return fail(GSVK_ERR_INVALID, "sv_create: %s has %zu channels, expected %d", p.c_str(),
                g.size(), c);
  std::vector<double> d(3 * static_cast<size_t>(c));
  for (int i = 0; i < c; ++i) {
    d[3 * i] = static_cast<double>(g[i]) / std::sqrt(static_cast<double>(var[i]) + 1e-5);
    d[3 * i + 1] = static_cast<double>(mu[i]);
    d[3 * i + 2] = static_cast<double>(b[i]);
  }
  return upload(h, out, d);
}

// load_conv_w (sv.cpp:97-128): the fp16 copy, else the fp32 copy rounded.
int load_conv(gsvk_sv* h, const TensorMap& m, const std::string& n, int co, int ci, int k,
              SvConv* c) {
  const gsvk_gsv_tensor* t = find(m, n);
  if (!t) return missing(n);
  const uint64_t numel = static_cast<uint64_t>(co) * ci * k * k;
  if (t->numel != numel)
    return fail(GSVK_ERR_INVALID, "sv_create: %s has %llu elements, expected %llu", n.c_str(),
                (unsigned long long)t->numel, (unsigned long long)numel);
  std::vector<uint16_t> w(numel);
  for (size_t i = 0; i < w.size(); ++i)
    w[i] = t->f16 ? t->f16[i] : __half_as_ushort(__float2half_rn(t->f32[i]));
  c->co = co, c->ci = ci, c->k = k;
  return upload(h, &c->w, w);
}

int load_aff(gsvk_sv* h, const TensorMap& m, const std::string& p, int ch, SvAffD* a) {
  const gsvk_gsv_tensor* t = find(m, p + "0.weight");
  if (!t) return missing(p + "0.weight");
  a->ch = ch;
  a->inter = static_cast<int>(t->numel / (2 * static_cast<uint64_t>(ch)));
  if (a->inter <= 0) return fail(GSVK_ERR_INVALID, "sv_create: bad %s0.weight", p.c_str());
  std::vector<float> b1, b2;
  int rc = load_conv(h, m, p + "0.weight", a->inter, 2 * ch, 1, &a->w1);
  if (!rc) rc = load_conv(h, m, p + "3.weight", ch, a->inter, 1, &a->w2);
  if (!rc) rc = vec_any(m, p + "0.bias", &b1);
  if (!rc) rc = vec_any(m, p + "3.bias", &b2);
  if (!rc && (static_cast<int>(b1.size()) != a->inter || static_cast<int>(b2.size()) != ch))
    rc = fail(GSVK_ERR_INVALID, "sv_create: %s biases mis-sized", p.c_str());
  if (!rc) rc = upload(h, &a->b1, b1);
  if (!rc) rc = upload(h, &a->b2, b2);
  if (!rc) rc = load_bn(h, m, p + "1", a->inter, &a->bn1);
  if (!rc) rc = load_bn(h, m, p + "4", ch, &a->bn2);
  return rc;
}

// load_block (sv.cpp:646-760) with the stage table of sv.cpp:791-795.
int load_block(gsvk_sv* h, const TensorMap& m, int l, int i, bool aff, int stride, int c_in,
               SvBlockD* b) {
  const std::string p = "layer" + std::to_string(l) + "." + std::to_string(i) + ".";
  const gsvk_gsv_tensor* c0 = find(m, p + "convs.0.weight");
  const gsvk_gsv_tensor* b3 = find(m, p + "bn3.weight");
  if (!c0) return missing(p + "convs.0.weight");
  if (!b3) return missing(p + "bn3.weight");
  b->aff = aff;
  b->stride = stride;
  b->c_in = c_in;
  b->width = c0->rank ? static_cast<int>(c0->dims[0]) : 0;
  b->exp = static_cast<int>(b3->numel);
  const int co1 = b->width * b->scale;
  if (b->width <= 0) return fail(GSVK_ERR_INVALID, "sv_create: bad %sconvs.0.weight", p.c_str());
  int rc = load_conv(h, m, p + "conv1.weight", co1, c_in, 1, &b->conv1);
  if (!rc) rc = load_bn(h, m, p + "bn1", co1, &b->bn1);
  b->convs.resize(b->scale);
  b->bns.resize(b->scale);
  for (int j = 0; j < b->scale && !rc; ++j) {
    rc = load_conv(h, m, p + "convs." + std::to_string(j) + ".weight", b->width, b->width, 3,
                   &b->convs[j]);
    if (!rc) rc = load_bn(h, m, p + "bns." + std::to_string(j), b->width, &b->bns[j]);
  }
  if (!rc && find(m, p + "convs." + std::to_string(b->scale) + ".weight"))
    rc = fail(GSVK_ERR_INVALID, "sv_create: %s has more than %d convs", p.c_str(), b->scale);
  if (!rc) rc = load_conv(h, m, p + "conv3.weight", b->exp, co1, 1, &b->conv3);
  if (!rc) rc = load_bn(h, m, p + "bn3", b->exp, &b->bn3);
  if (aff) {
    b->fuses.resize(b->scale - 1);
    for (int j = 0; j < b->scale - 1 && !rc; ++j)
      rc = load_aff(h, m, p + "fuse_models." + std::to_string(j) + ".local_att.", b->width,
                    &b->fuses[j]);
  }
  b->has_sc = find(m, p + "shortcut.0.weight") != nullptr;
  if (!rc && b->has_sc) {
    rc = load_conv(h, m, p + "shortcut.0.weight", b->exp, c_in, 1, &b->sc);
    if (!rc) rc = load_bn(h, m, p + "shortcut.1", b->exp, &b->sc_bn);
  }
  if (!rc && !b->has_sc && (stride != 1 || c_in != b->exp))
    rc = fail(GSVK_ERR_INVALID, "sv_create: %s changes shape without a shortcut", p.c_str());
  return rc;
}

// out[c_out][S] = W[c_out][K] . cols[S][K]^T.  (A per-channel bias is a
// per-row term here, which the GEMM epilogue's per-column bias cannot
// express; the kernel after the GEMM adds it.)
int gemm_cols(const SvConv& c, const uint16_t* cols, int S, float* out, cudaStream_t st) {
  gsvk_gemm_args g{};
  const size_t K = static_cast<size_t>(c.ci) * c.k * c.k;
  g.a = c.w;
  g.lda = K;
  g.b = cols;
  g.ldb = K;
  g.M = static_cast<size_t>(c.co);
  g.N = static_cast<size_t>(S);
  g.K = K;
  g.c = out;
  g.ldc = static_cast<size_t>(S);
  g.act = GSVK_ACT_NONE;
  g.alpha = 1.f;
  // B is the im2col just written by the previous kernel: no early B loads
  return gemm_ex_run(&g, st, false);
}

// conv2d_f16 (sv.cpp:196-258): out [c_out][oh*ow].
int conv2d(gsvk_sv* h, const SvConv& c, const float* in, int hh, int ww, int stride, int pad,
           float* out, cudaStream_t st) {
  const int oh = (hh + 2 * pad - c.k) / stride + 1, ow = (ww + 2 * pad - c.k) / stride + 1;
  const int S = oh * ow;
  if (c.k == 1 && stride == 1 && pad == 0) {
    dim3 grid((S + 31) / 32, (c.ci + 31) / 32);
    transpose_f16_kernel<<<grid, 256, 0, st>>>(in, in, c.ci, c.ci, S, h->cols);
    if (int rc = check_launch("transpose_f16_kernel")) return rc;
  } else {
    im2col2d_kernel<uint16_t><<<grid_for(static_cast<long long>(S) * c.ci), 256, 0, st>>>(
        in, c.ci, hh, ww, c.k, c.k, stride, pad, ow, S, h->cols);
    if (int rc = check_launch("im2col2d_kernel")) return rc;
  }
  return gemm_cols(c, h->cols, S, out, st);
}

int bn_act(const float* x, int C, int S, const double* bn, int act, float* y, float* y2,
           cudaStream_t st, const float* bias = nullptr) {
  bn_act_kernel<<<grid_for(static_cast<long long>(C) * S), 256, 0, st>>>(x, bias, C, S, bn, act,
                                                                          y, y2);
  return check_launch("bn_act_kernel");
}

// Aff::apply (sv.cpp:445-521); out may alias x.
int aff_apply(gsvk_sv* h, const SvAffD& a, const float* x, const float* ds, float* out, int S,
              cudaStream_t st) {
  dim3 g1((S + 31) / 32, (2 * a.ch + 31) / 32);
  transpose_f16_kernel<<<g1, 256, 0, st>>>(x, ds, a.ch, 2 * a.ch, S, h->cols);
  int rc = check_launch("transpose_f16_kernel");
  if (!rc) rc = gemm_cols(a.w1, h->cols, S, h->att, st);
  if (!rc) rc = bn_act(h->att, a.inter, S, a.bn1, kActSilu, h->att, nullptr, st, a.b1);
  if (!rc) {
    dim3 g2((S + 31) / 32, (a.inter + 31) / 32);
    transpose_f16_kernel<<<g2, 256, 0, st>>>(h->att, h->att, a.inter, a.inter, S, h->cols);
    rc = check_launch("transpose_f16_kernel");
  }
  if (!rc) rc = gemm_cols(a.w2, h->cols, S, h->at, st);
  if (!rc) {
    aff_combine_kernel<<<grid_for(static_cast<long long>(a.ch) * S), 256, 0, st>>>(
        h->at, a.b2, a.bn2, x, ds, a.ch, S, out);
    rc = check_launch("aff_combine_kernel");
  }
  return rc;
}

// Block::apply (sv.cpp:523-644): in [c_in][hh][ww] -> out [exp][h'][w'].
int block_apply(gsvk_sv* h, const SvBlockD& b, const float* in, int& hh, int& ww, float* out,
                cudaStream_t st) {
  const int co1 = b.width * b.scale, h_in = hh, w_in = ww;
  int rc = conv2d(h, b.conv1, in, hh, ww, b.stride, 0, h->c1, st);
  hh = (hh - 1) / b.stride + 1;
  ww = (ww - 1) / b.stride + 1;
  const int S = hh * ww;
  if (!rc) rc = bn_act(h->c1, co1, S, b.bn1, kActRelu20, h->c1, nullptr, st);
  const size_t part = static_cast<size_t>(b.width) * S;
  for (int i = 0; i < b.scale && !rc; ++i) {
    const float* chunk = h->c1 + i * part;
    if (i > 0) {
      if (b.aff) {
        rc = aff_apply(h, b.fuses[i - 1], h->sp, chunk, h->sp, S, st);
      } else {
        add_inplace_kernel<<<grid_for(static_cast<long long>(part)), 256, 0, st>>>(
            h->sp, chunk, static_cast<long long>(part));
        rc = check_launch("add_inplace_kernel");
      }
    }
    float* slot = h->tmp2 + i * part;
    if (!rc) rc = conv2d(h, b.convs[i], i == 0 ? chunk : h->sp, hh, ww, 1, 1, slot, st);
    if (!rc) rc = bn_act(slot, b.width, S, b.bns[i], kActRelu20, slot, h->sp, st);
  }
  if (!rc) rc = conv2d(h, b.conv3, h->tmp2, hh, ww, 1, 0, out, st);
  const float* res = in;
  if (!rc && b.has_sc) {
    rc = conv2d(h, b.sc, in, h_in, w_in, b.stride, 0, h->sc, st);
    res = h->sc;
  }
  if (!rc) {
    block_tail_kernel<<<grid_for(static_cast<long long>(b.exp) * S), 256, 0, st>>>(
        out, b.bn3, res, b.has_sc ? b.sc_bn : nullptr, b.exp, S, out);
    rc = check_launch("block_tail_kernel");
  }
  return rc;
}

int create_impl(gsvk_sv* h, const TensorMap& m) {
  const int F = h->cfg.n_mels;
  std::vector<float> w0;
  int rc = vec_any(m, "conv1.weight", &w0);
  if (rc) return rc;
  if (w0.empty() || w0.size() % 9) return fail(GSVK_ERR_INVALID, "sv_create: stem conv is not [c][1][3][3]");
  h->m_ch = static_cast<int>(w0.size() / 9);
  rc = upload(h, &h->stem_w, w0);
  if (!rc) rc = load_bn(h, m, "bn1", h->m_ch, &h->stem_bn);
  struct Def {
    int blocks, stride;
    bool aff;
  };
  const Def defs[4] = {{3, 1, false}, {4, 2, false}, {6, 2, true}, {3, 2, true}};
  int c = h->m_ch;
  // workspace sizes: spatial size per stage, largest products
  const size_t S1 = static_cast<size_t>(F) * h->cfg.max_frames;
  size_t act = S1 * c, c1 = 0, cols = S1 * 9, att = 0, at = 0;
  int hh = F, ww = static_cast<int>(h->cfg.max_frames);
  for (int l = 0; l < 4 && !rc; ++l) {
    h->blocks[l].resize(defs[l].blocks);
    for (int i = 0; i < defs[l].blocks && !rc; ++i) {
      SvBlockD& b = h->blocks[l][i];
      const int stride = i == 0 ? defs[l].stride : 1;
      rc = load_block(h, m, l + 1, i, defs[l].aff, stride, c, &b);
      if (rc) break;
      hh = (hh - 1) / stride + 1;
      ww = (ww - 1) / stride + 1;
      const size_t s = static_cast<size_t>(hh) * ww;
      const size_t co1 = static_cast<size_t>(b.width) * b.scale;
      c1 = std::max(c1, co1 * s);
      act = std::max(act, static_cast<size_t>(b.exp) * s);
      cols = std::max({cols, s * c, s * b.width * 9, s * co1});
      for (const SvAffD& a : b.fuses) {
        cols = std::max({cols, s * 2 * a.ch, s * a.inter});
        att = std::max(att, static_cast<size_t>(a.inter) * s);
        at = std::max(at, static_cast<size_t>(a.ch) * s);
      }
      c = b.exp;
    }
    if (l == 2) h->c3 = c;
  }
  if (rc) return rc;
  h->c4 = c;
  const int h4 = hh, w4 = ww;
  // layer3_ds (k3 s2 p1) on the layer-3 output and fuse34
  rc = load_conv(h, m, "layer3_ds.weight", h->c4, h->c3, 3, &h->l3ds);
  if (!rc) rc = load_aff(h, m, "fuse34.local_att.", h->c4, &h->fuse34);
  if (rc) return rc;
  const size_t S4 = static_cast<size_t>(h4) * w4;
  cols = std::max({cols, S4 * h->c3 * 9, S4 * 2 * h->c4, S4 * h->fuse34.inter});
  att = std::max(att, static_cast<size_t>(h->fuse34.inter) * S4);
  at = std::max(at, static_cast<size_t>(h->c4) * S4);
  rc = dev_alloc(h, reinterpret_cast<void**>(&h->img), S1 * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->A), act * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->B), act * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->sc), act * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->c1), c1 * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->tmp2), c1 * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->sp), c1 * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->ds), static_cast<size_t>(h->c4) * S4 * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->att), att * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->at), at * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->cols32), S1 * 9 * 4);
  if (!rc) rc = dev_alloc(h, reinterpret_cast<void**>(&h->cols), cols * 2);
  return rc;
}

}  // namespace

extern "C" {

int gsvk_sv_destroy(gsvk_sv_t h) {
  if (!h) return GSVK_OK;
  for (void* p : h->allocs) cudaFree(p);
  delete h;
  return GSVK_OK;
}

int gsvk_sv_create(const gsvk_sv_config* cfg, const gsvk_gsv_tensor* tensors, size_t n,
                   gsvk_sv_t* out) {
  if (!cfg || !tensors || !out) return fail(GSVK_ERR_INVALID, "sv_create: null argument");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  if (cfg->n_mels < 8 || cfg->max_frames < 8 || cfg->max_frames > 100000)
    return fail(GSVK_ERR_INVALID, "sv_create: n_mels >= 8 and 8 <= max_frames <= 100000");
  TensorMap m;
  for (size_t i = 0; i < n; ++i)
    if (tensors[i].name) m[tensors[i].name] = &tensors[i];
  auto* h = new gsvk_sv();
  h->cfg = *cfg;
  if (int rc = create_impl(h, m)) {
    gsvk_sv_destroy(h);
    return rc;
  }
  *out = h;
  return GSVK_OK;
}

int gsvk_sv_create_from_gsv(gsvk_gsv_t f, const gsvk_sv_config* cfg, gsvk_sv_t* out) {
  if (!f || !out) return fail(GSVK_ERR_INVALID, "sv_create_from_gsv: null argument");
  const size_t n = gsvk_gsv_count(f);
  std::vector<gsvk_gsv_tensor> t(n);
  for (size_t i = 0; i < n; ++i)
    if (int rc = gsvk_gsv_tensor_at(f, i, &t[i])) return rc;
  return gsvk_sv_create(cfg, t.data(), n, out);
}

size_t gsvk_sv_embedding_size(gsvk_sv_t h) {
  if (!h) return 0;
  int f = h->cfg.n_mels;
  for (int l = 0; l < 4; ++l)
    for (const SvBlockD& b : h->blocks[l]) f = (f - 1) / b.stride + 1;
  return static_cast<size_t>(h->c4) * f;
}

int gsvk_sv_forward(gsvk_sv_t h, const float* fbank, size_t frames, float* emb,
                    gsvk_stream_t stream) {
  if (!h || !fbank || !emb) return fail(GSVK_ERR_INVALID, "sv_forward: null argument");
  if (frames < 1 || frames > h->cfg.max_frames)
    return fail(GSVK_ERR_INVALID, "sv_forward: %zu frames outside 1..%zu", frames,
                h->cfg.max_frames);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int F = h->cfg.n_mels, T = static_cast<int>(frames);
  const int S1 = F * T;
  fbank_to_image_kernel<<<grid_for(S1), 256, 0, st>>>(fbank, T, F, h->img);
  int rc = check_launch("fbank_to_image_kernel");
  // stem: conv2d in fp32 (sv.cpp:171-194, 810-814), BN, ReLU
  if (!rc) {
    im2col2d_kernel<float><<<grid_for(S1), 256, 0, st>>>(h->img, 1, F, T, 3, 3, 1, 1, T, S1,
                                                         h->cols32);
    rc = check_launch("im2col2d_kernel");
  }
  if (!rc)
    rc = gsvk_sgemm('N', 'T', h->m_ch, S1, 9, 1.f, h->stem_w, 9, h->cols32, 9, 0.f, h->B, S1,
                    stream);
  if (!rc) rc = bn_act(h->B, h->m_ch, S1, h->stem_bn, kActRelu, h->A, nullptr, st);
  int hh = F, ww = T;
  float* cur = h->A;
  float* nxt = h->B;
  for (int l = 0; l < 4 && !rc; ++l) {
    for (size_t i = 0; i < h->blocks[l].size() && !rc; ++i) {
      rc = block_apply(h, h->blocks[l][i], cur, hh, ww, nxt, st);
      std::swap(cur, nxt);
    }
    if (l == 2 && !rc)  // layer3_ds on the layer-3 output (sv.cpp:852-862)
      rc = conv2d(h, h->l3ds, cur, hh, ww, 2, 1, h->ds, st);
  }
  const int S4 = hh * ww;
  // fuse34 on (layer-4 output, ds), then the mean over time
  if (!rc) rc = aff_apply(h, h->fuse34, cur, h->ds, nxt, S4, st);
  if (!rc) {
    const int rows = h->c4 * hh;
    mean_rows_kernel<<<(rows + 7) / 8, 256, 0, st>>>(nxt, rows, ww, emb);
    rc = check_launch("mean_rows_kernel");
  }
  return rc;
}

}  // extern "C"
