// sv.cu — the SV speaker encoder (ERes2NetV2 w24 s4 e4) on the device
// (GPT-SoVITS-native src/encoder/sv.cpp:130-885, the default path): the
// fp32 stem conv, four Res2Net stages (1x1 / 3x3 / strided convs, BatchNorm
// in the fp64 chain, relu20, hierarchical splits with AFF fusion in stages
// 3-4), layer3_ds, the fuse34 AFF and the mean over time.
//
// Activations are channels-last [H*W][C] fp32 (the transpose of the
// reference's channel-major [C][H][W]), with an fp16 copy where a conv reads
// them.  A convolution is one tensor-core GEMM out[S][c_out] = A[S][K] .
// W[c_out][K]^T (fp16 operands, fp32 accumulate: the reference's conv2d_f16
// arithmetic, summed in another order):
//   - 1x1 stride 1: A is the fp16 activation itself (no copy);
//   - 1x1 stride 2: A gathers every other pixel's channel row;
//   - 3x3: A = im2col with tap-major columns (ky*3 + kx)*c_in + c, so each
//     tap is one contiguous channel row; the weights are permuted to that
//     column order once at create.
// Per-channel biases (the AFF convs) are per-column terms here and go in the
// GEMM epilogue; BatchNorm, relu20, SiLU and the residual adds run in small
// element-wise kernels.  The stem conv (c_in = 1, K = 9) keeps fp32 operands
// on the sgemm kernel, as the reference's conv2d does.
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
// double operation rounded separately; p = (a, mu, beta).
__device__ __forceinline__ float bn64(float x, const double* p) {
  return static_cast<float>(
      __dadd_rn(__dmul_rn(__dsub_rn(static_cast<double>(x), p[1]), p[0]), p[2]));
}

__device__ __forceinline__ float act_apply(float v, int act) {
  if (act == kActRelu) return v < 0.f ? 0.f : v;
  if (act == kActRelu20) return relu20(v);
  if (act == kActSilu) return __fdiv_rn(v, __fadd_rn(1.f, expf(-v)));  // kern.cpp:80-83
  return v;
}

// cols[s][(ky*kw + kx)*c + ch] = f16(x[(iy*w + ix)*ldx + ch]), zero outside
// the image (iy = oy*stride - pad + ky, ix likewise).  One thread per 8
// channels of one (pixel, tap): two 16-byte loads, one 16-byte store (c, ldx
// multiples of 8 and 4, x 16-byte aligned).
__global__ void im2col_rows_kernel(const float* __restrict__ x, int ldx, int c, int h, int w,
                                   int kh, int kw, int stride, int pad, int ow, int S,
                                   uint16_t* __restrict__ cols) {
  const int c8 = c >> 3, taps = kh * kw;
  const long long n = static_cast<long long>(S) * taps * c8;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / c8;
    const int g = static_cast<int>(e - r * c8);
    const int s = static_cast<int>(r / taps);
    const int tap = static_cast<int>(r - static_cast<long long>(s) * taps);
    const int ky = tap / kw, kx = tap - ky * kw;
    const int oy = s / ow, ox = s - oy * ow;
    const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
      const float4* src = reinterpret_cast<const float4*>(
          x + (static_cast<size_t>(iy) * w + ix) * ldx + 8 * g);
      const float4 a = src[0], b = src[1];
      o.x = f2h(a.x) | (static_cast<uint32_t>(f2h(a.y)) << 16);
      o.y = f2h(a.z) | (static_cast<uint32_t>(f2h(a.w)) << 16);
      o.z = f2h(b.x) | (static_cast<uint32_t>(f2h(b.y)) << 16);
      o.w = f2h(b.z) | (static_cast<uint32_t>(f2h(b.w)) << 16);
    }
    *reinterpret_cast<uint4*>(cols + static_cast<size_t>(s) * taps * c + tap * c + 8 * g) = o;
  }
}

// The stem's fp32 cols[s][ky*3 + kx] of the one-channel F x T image (the
// fbank [T][F] read transposed: pixel (f, t) = fb[t][f]).
__global__ void stem_cols_kernel(const float* __restrict__ fb, int T, int F,
                                 float* __restrict__ cols) {
  const long long n = static_cast<long long>(F) * T * 9;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long s = e / 9;
    const int tap = static_cast<int>(e - s * 9);
    const int f = static_cast<int>(s / T), t = static_cast<int>(s - static_cast<long long>(f) * T);
    const int iy = f - 1 + tap / 3, ix = t - 1 + tap % 3;
    cols[e] =
        (iy >= 0 && iy < F && ix >= 0 && ix < T) ? fb[static_cast<size_t>(ix) * F + iy] : 0.f;
  }
}

// y = act(BN(x)) on rows [S][C] (x row stride ldx), into an fp32 and/or an
// fp16 output with their own row strides.  One thread per 4 channels of a
// row (C and the strides multiples of 4, 16-byte aligned rows).
__global__ void bn_act_kernel(const float* x, int ldx, int C, int S, const double* __restrict__ bn,
                              int act, float* y, int ldy, uint16_t* y16, int ldy16) {
  const int C4 = C >> 2;
  const long long n = static_cast<long long>(C4) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(e / C4);
    const int c = 4 * static_cast<int>(e - static_cast<long long>(s) * C4);
    const float4 v = *reinterpret_cast<const float4*>(x + static_cast<size_t>(s) * ldx + c);
    float4 r;
    r.x = act_apply(bn64(v.x, bn + 3 * c), act);
    r.y = act_apply(bn64(v.y, bn + 3 * c + 3), act);
    r.z = act_apply(bn64(v.z, bn + 3 * c + 6), act);
    r.w = act_apply(bn64(v.w, bn + 3 * c + 9), act);
    if (y) *reinterpret_cast<float4*>(y + static_cast<size_t>(s) * ldy + c) = r;
    if (y16) {
      uint2 o;
      o.x = f2h(r.x) | (static_cast<uint32_t>(f2h(r.y)) << 16);
      o.y = f2h(r.z) | (static_cast<uint32_t>(f2h(r.w)) << 16);
      *reinterpret_cast<uint2*>(y16 + static_cast<size_t>(s) * ldy16 + c) = o;
    }
  }
}

// Block tail (sv.cpp:612-643): out = relu20(BN3(a) + (bnsc ? BNsc(b) : b)),
// fp32 and fp16.
__global__ void block_tail_kernel(const float* a, const double* __restrict__ bn3,
                                  const float* __restrict__ b, const double* __restrict__ bnsc,
                                  int C, int S, float* out, uint16_t* __restrict__ out16) {
  const long long n = static_cast<long long>(C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e % C);
    const float u = bn64(a[e], bn3 + 3 * c);
    const float r = bnsc ? bn64(b[e], bnsc + 3 * c) : b[e];
    const float v = relu20(__fadd_rn(u, r));
    out[e] = v;
    out16[e] = f2h(v);
  }
}

// y[s][c] += x[s][c] (row strides ldy, ldx): the Res2Net split sum.
__global__ void add_rows_kernel(float* y, int ldy, const float* __restrict__ x, int ldx, int C,
                                int S) {
  const long long n = static_cast<long long>(C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(e / C), c = static_cast<int>(e - static_cast<long long>(s) * C);
    float& d = y[static_cast<size_t>(s) * ldy + c];
    d = __fadd_rn(d, x[static_cast<size_t>(s) * ldx + c]);
  }
}

// AFF input: cat[s] = f16([x[s][0..C) | ds[s][0..C)]).
__global__ void aff_cat_kernel(const float* __restrict__ x, int ldx, const float* __restrict__ ds,
                               int ldd, int C, int S, uint16_t* __restrict__ cat) {
  const long long n = static_cast<long long>(2 * C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(e / (2 * C));
    const int c = static_cast<int>(e - static_cast<long long>(s) * 2 * C);
    cat[e] = f2h(c < C ? x[static_cast<size_t>(s) * ldx + c]
                       : ds[static_cast<size_t>(s) * ldd + c - C]);
  }
}

// AFF output (sv.cpp:506-520): t = tanh(BN2(at)); out = x (1 + t) + ds (1 - t).
__global__ void aff_combine_kernel(const float* __restrict__ at, const double* __restrict__ bn,
                                   const float* x, int ldx, const float* __restrict__ ds, int ldd,
                                   int C, int S, float* out, int ldo) {
  const long long n = static_cast<long long>(C) * S;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(e / C), c = static_cast<int>(e - static_cast<long long>(s) * C);
    const float t = tanhf(bn64(at[e], bn + 3 * c));
    const float xv = x[static_cast<size_t>(s) * ldx + c];
    const float dv = ds[static_cast<size_t>(s) * ldd + c];
    out[static_cast<size_t>(s) * ldo + c] =
        __fadd_rn(__fmul_rn(xv, __fadd_rn(1.f, t)), __fmul_rn(dv, __fsub_rn(1.f, t)));
  }
}

// emb[c*h + fy] = float(sum_t double(x[(fy*w + t)][c]) / w), summed in time
// order (sv.cpp:870-879); one thread per (c, fy), consecutive threads on
// consecutive channels.
__global__ void mean_time_kernel(const float* __restrict__ x, int C, int h, int w,
                                 float* __restrict__ emb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= C * h) return;
  const int fy = i / C, c = i - fy * C;
  double acc = 0.0;
  for (int t = 0; t < w; ++t)
    acc += static_cast<double>(x[(static_cast<size_t>(fy) * w + t) * C + c]);
  emb[static_cast<size_t>(c) * h + fy] = static_cast<float>(acc / w);
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
  uint16_t* w = nullptr;  // [c_out][k*k*c_in], tap-major columns
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
  // workspaces (channels-last rows)
  float* X[2] = {nullptr, nullptr};
  uint16_t* X16[2] = {nullptr, nullptr};
  float *c1 = nullptr, *sp = nullptr, *cv = nullptr, *sc = nullptr, *ds = nullptr;
  float *att = nullptr, *at = nullptr, *cols32 = nullptr, *fused = nullptr;
  uint16_t *tmp16 = nullptr, *cols = nullptr, *att16 = nullptr;
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
int alloc_n(gsvk_sv* h, T** p, size_t n) {
  return dev_alloc(h, reinterpret_cast<void**>(p), n * sizeof(T));
}

template <typename T>
int upload(gsvk_sv* h, T** dst, const std::vector<T>& src) {
  if (int rc = alloc_n(h, dst, src.size())) return rc;
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

// load_conv_w (sv.cpp:97-128): the fp16 copy, else the fp32 copy rounded;
// [co][ci][k][k] -> [co][(ky*k + kx)*ci + c] (the im2col's column order).
int load_conv(gsvk_sv* h, const TensorMap& m, const std::string& n, int co, int ci, int k,
              SvConv* cv) {
  const gsvk_gsv_tensor* t = find(m, n);
  if (!t) return missing(n);
  const uint64_t numel = static_cast<uint64_t>(co) * ci * k * k;
  if (t->numel != numel)
    return fail(GSVK_ERR_INVALID, "sv_create: %s has %llu elements, expected %llu", n.c_str(),
                (unsigned long long)t->numel, (unsigned long long)numel);
  std::vector<uint16_t> w(numel);
  const size_t K = static_cast<size_t>(ci) * k * k;
  for (int o = 0; o < co; ++o)
    for (int c = 0; c < ci; ++c)
      for (int tap = 0; tap < k * k; ++tap) {
        const size_t src = (static_cast<size_t>(o) * ci + c) * k * k + tap;
        w[o * K + static_cast<size_t>(tap) * ci + c] =
            t->f16 ? t->f16[src] : __half_as_ushort(__float2half_rn(t->f32[src]));
      }
  cv->co = co, cv->ci = ci, cv->k = k;
  return upload(h, &cv->w, w);
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

// out[S][c_out] = A[S][K] . W[c_out][K]^T (+ bias[c_out]); W is the static
// operand.
int gemm_rows(const SvConv& c, const uint16_t* a, int S, const float* bias, float* out,
              cudaStream_t st) {
  gsvk_gemm_args g{};
  const size_t K = static_cast<size_t>(c.ci) * c.k * c.k;
  g.a = a;
  g.lda = K;
  g.b = c.w;
  g.ldb = K;
  g.M = static_cast<size_t>(S);
  g.N = static_cast<size_t>(c.co);
  g.K = K;
  g.bias = bias;
  g.c = out;
  g.ldc = static_cast<size_t>(c.co);
  g.act = GSVK_ACT_NONE;
  g.alpha = 1.f;
  return gemm_ex_run(&g, st, true);
}

// conv2d_f16 (sv.cpp:196-258) on rows: x fp32 [hh*ww][ldx] (channels
// [0, c.ci)) or, for a 1x1 stride-1 conv, its fp16 copy x16 [hh*ww][c.ci];
// out [oh*ow][c.co].
int conv2d(gsvk_sv* h, const SvConv& c, const float* x, int ldx, const uint16_t* x16, int hh,
           int ww, int stride, int pad, const float* bias, float* out, cudaStream_t st) {
  const int oh = (hh + 2 * pad - c.k) / stride + 1, ow = (ww + 2 * pad - c.k) / stride + 1;
  const int S = oh * ow;
  const uint16_t* a = x16;
  if (!(c.k == 1 && stride == 1 && pad == 0 && x16)) {
    if (c.ci % 8 || ldx % 4 || reinterpret_cast<uintptr_t>(x) % 16)
      return fail(GSVK_ERR_ALIGN, "sv conv: channels not a multiple of 8 or unaligned rows");
    const long long n = static_cast<long long>(S) * c.k * c.k * (c.ci / 8);
    im2col_rows_kernel<<<grid_for(n), 256, 0, st>>>(x, ldx, c.ci, hh, ww, c.k, c.k, stride, pad,
                                                    ow, S, h->cols);
    if (int rc = check_launch("im2col_rows_kernel")) return rc;
    a = h->cols;
  }
  return gemm_rows(c, a, S, bias, out, st);
}

int bn_act(const float* x, int ldx, int C, int S, const double* bn, int act, float* y, int ldy,
           uint16_t* y16, int ldy16, cudaStream_t st) {
  if (C % 4 || ldx % 4 || ldy % 4 || ldy16 % 4 ||
      (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) % 16 ||
      reinterpret_cast<uintptr_t>(y16) % 8)
    return fail(GSVK_ERR_ALIGN, "sv batch norm: channels not a multiple of 4 or unaligned rows");
  bn_act_kernel<<<grid_for(static_cast<long long>(C / 4) * S), 256, 0, st>>>(
      x, ldx, C, S, bn, act, y, ldy, y16, ldy16);
  return check_launch("bn_act_kernel");
}

// Aff::apply (sv.cpp:445-521) on rows; out may alias x.
int aff_apply(gsvk_sv* h, const SvAffD& a, const float* x, int ldx, const float* ds, int ldd,
              float* out, int ldo, int S, cudaStream_t st) {
  aff_cat_kernel<<<grid_for(static_cast<long long>(2 * a.ch) * S), 256, 0, st>>>(
      x, ldx, ds, ldd, a.ch, S, h->cols);
  int rc = check_launch("aff_cat_kernel");
  if (!rc) rc = gemm_rows(a.w1, h->cols, S, a.b1, h->att, st);
  if (!rc)
    rc = bn_act(h->att, a.inter, a.inter, S, a.bn1, kActSilu, nullptr, 0, h->att16, a.inter, st);
  if (!rc) rc = gemm_rows(a.w2, h->att16, S, a.b2, h->at, st);
  if (!rc) {
    aff_combine_kernel<<<grid_for(static_cast<long long>(a.ch) * S), 256, 0, st>>>(
        h->at, a.bn2, x, ldx, ds, ldd, a.ch, S, out, ldo);
    rc = check_launch("aff_combine_kernel");
  }
  return rc;
}

// Block::apply (sv.cpp:523-644): in / in16 [hh*ww][c_in] -> out / out16
// [h'*w'][exp].
int block_apply(gsvk_sv* h, const SvBlockD& b, const float* in, const uint16_t* in16, int& hh,
                int& ww, float* out, uint16_t* out16, cudaStream_t st) {
  const int co1 = b.width * b.scale, h_in = hh, w_in = ww;
  int rc = conv2d(h, b.conv1, in, b.c_in, in16, hh, ww, b.stride, 0, nullptr, h->c1, st);
  hh = (hh - 1) / b.stride + 1;
  ww = (ww - 1) / b.stride + 1;
  const int S = hh * ww, wd = b.width;
  if (!rc) rc = bn_act(h->c1, co1, co1, S, b.bn1, kActRelu20, h->c1, co1, nullptr, 0, st);
  for (int i = 0; i < b.scale && !rc; ++i) {
    const float* chunk = h->c1 + i * wd;  // channels [i*wd, (i+1)*wd) of c1, row stride co1
    if (i > 0) {
      if (b.aff) {
        rc = aff_apply(h, b.fuses[i - 1], h->sp, wd, chunk, co1, h->sp, wd, S, st);
      } else {
        add_rows_kernel<<<grid_for(static_cast<long long>(wd) * S), 256, 0, st>>>(
            h->sp, wd, chunk, co1, wd, S);
        rc = check_launch("add_rows_kernel");
      }
    }
    if (!rc)
      rc = i == 0 ? conv2d(h, b.convs[i], chunk, co1, nullptr, hh, ww, 1, 1, nullptr, h->cv, st)
                  : conv2d(h, b.convs[i], h->sp, wd, nullptr, hh, ww, 1, 1, nullptr, h->cv, st);
    // BN + relu20 -> sp (the next split's input) and slot i of conv3's input
    if (!rc)
      rc = bn_act(h->cv, wd, wd, S, b.bns[i], kActRelu20, h->sp, wd, h->tmp16 + i * wd, co1, st);
  }
  if (!rc) rc = gemm_rows(b.conv3, h->tmp16, S, nullptr, out, st);
  const float* res = in;
  if (!rc && b.has_sc) {
    rc = conv2d(h, b.sc, in, b.c_in, in16, h_in, w_in, b.stride, 0, nullptr, h->sc, st);
    res = h->sc;
  }
  if (!rc) {
    block_tail_kernel<<<grid_for(static_cast<long long>(b.exp) * S), 256, 0, st>>>(
        out, b.bn3, res, b.has_sc ? b.sc_bn : nullptr, b.exp, S, out, out16);
    rc = check_launch("block_tail_kernel");
  }
  return rc;
}

int create_impl(gsvk_sv* h, const TensorMap& m) {
  const int F = h->cfg.n_mels;
  std::vector<float> w0;
  int rc = vec_any(m, "conv1.weight", &w0);
  if (rc) return rc;
  if (w0.empty() || w0.size() % 9)
    return fail(GSVK_ERR_INVALID, "sv_create: stem conv is not [c][1][3][3]");
  h->m_ch = static_cast<int>(w0.size() / 9);
  rc = upload(h, &h->stem_w, w0);
  if (!rc) rc = load_bn(h, m, "bn1", h->m_ch, &h->stem_bn);
  struct Def {
    int blocks, stride;
    bool aff;
  };
  const Def defs[4] = {{3, 1, false}, {4, 2, false}, {6, 2, true}, {3, 2, true}};
  int c = h->m_ch;
  const size_t S1 = static_cast<size_t>(F) * h->cfg.max_frames;
  size_t act = S1 * c, c1 = 0, wdS = 0, cols = 0, att = 0, at = 0;
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
      wdS = std::max(wdS, static_cast<size_t>(b.width) * s);
      act = std::max(act, static_cast<size_t>(b.exp) * s);
      cols = std::max({cols, s * b.width * 9, stride != 1 ? s * c : size_t{0}});
      for (const SvAffD& a : b.fuses) {
        cols = std::max(cols, s * 2 * a.ch);
        att = std::max(att, static_cast<size_t>(a.inter) * s);
        at = std::max(at, static_cast<size_t>(a.ch) * s);
      }
      c = b.exp;
    }
    if (l == 2) h->c3 = c;
  }
  if (rc) return rc;
  h->c4 = c;
  // layer3_ds (k3 s2 p1) on the layer-3 output and fuse34
  rc = load_conv(h, m, "layer3_ds.weight", h->c4, h->c3, 3, &h->l3ds);
  if (!rc) rc = load_aff(h, m, "fuse34.local_att.", h->c4, &h->fuse34);
  if (rc) return rc;
  const size_t S4 = static_cast<size_t>(hh) * ww;
  cols = std::max({cols, S4 * h->c3 * 9, S4 * 2 * h->c4});
  att = std::max(att, static_cast<size_t>(h->fuse34.inter) * S4);
  at = std::max(at, static_cast<size_t>(h->c4) * S4);
  for (int i = 0; i < 2 && !rc; ++i) {
    rc = alloc_n(h, &h->X[i], act);
    if (!rc) rc = alloc_n(h, &h->X16[i], act);
  }
  if (!rc) rc = alloc_n(h, &h->c1, c1);
  if (!rc) rc = alloc_n(h, &h->tmp16, c1);
  if (!rc) rc = alloc_n(h, &h->sp, wdS);
  if (!rc) rc = alloc_n(h, &h->cv, wdS);
  if (!rc) rc = alloc_n(h, &h->sc, act);
  if (!rc) rc = alloc_n(h, &h->ds, static_cast<size_t>(h->c4) * S4);
  if (!rc) rc = alloc_n(h, &h->fused, static_cast<size_t>(h->c4) * S4);
  if (!rc) rc = alloc_n(h, &h->att, att);
  if (!rc) rc = alloc_n(h, &h->att16, att);
  if (!rc) rc = alloc_n(h, &h->at, at);
  if (!rc) rc = alloc_n(h, &h->cols32, S1 * 9);
  if (!rc) rc = alloc_n(h, &h->cols, cols);
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
  const int F = h->cfg.n_mels, T = static_cast<int>(frames), S1 = F * T;
  // stem: conv2d in fp32 (sv.cpp:171-194, 805-814) as out[S][m_ch] = cols .
  // W^T on the sgemm kernel, then BN and ReLU
  stem_cols_kernel<<<grid_for(static_cast<long long>(S1) * 9), 256, 0, st>>>(fbank, T, F,
                                                                            h->cols32);
  int rc = check_launch("stem_cols_kernel");
  if (!rc)
    rc = gsvk_sgemm('N', 'T', S1, h->m_ch, 9, 1.f, h->cols32, 9, h->stem_w, 9, 0.f, h->X[1],
                    h->m_ch, stream);
  if (!rc)
    rc = bn_act(h->X[1], h->m_ch, h->m_ch, S1, h->stem_bn, kActRelu, h->X[0], h->m_ch, h->X16[0],
                h->m_ch, st);
  int hh = F, ww = T, cur = 0;
  for (int l = 0; l < 4 && !rc; ++l) {
    for (size_t i = 0; i < h->blocks[l].size() && !rc; ++i) {
      rc = block_apply(h, h->blocks[l][i], h->X[cur], h->X16[cur], hh, ww, h->X[1 - cur],
                       h->X16[1 - cur], st);
      cur = 1 - cur;
    }
    if (l == 2 && !rc)  // layer3_ds on the layer-3 output (sv.cpp:852-862)
      rc = conv2d(h, h->l3ds, h->X[cur], h->c3, nullptr, hh, ww, 2, 1, nullptr, h->ds, st);
  }
  const int S4 = hh * ww;
  // fuse34 on (layer-4 output, ds), then the mean over time
  if (!rc)
    rc = aff_apply(h, h->fuse34, h->X[cur], h->c4, h->ds, h->c4, h->fused, h->c4, S4, st);
  if (!rc) {
    const int n = h->c4 * hh;
    mean_time_kernel<<<(n + 255) / 256, 256, 0, st>>>(h->fused, h->c4, hh, ww, emb);
    rc = check_launch("mean_time_kernel");
  }
  return rc;
}

}  // extern "C"
