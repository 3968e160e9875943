// sovits_latent.cu — the SoVITS latent path on the device
// (GPT-SoVITS-native src/sovits/sovits_engine.hpp:48-93, steps 1-5): RVQ
// decode and nearest x2 (quantizer.hpp:26-38), the TextEncoder (enc_p.hpp:
// ssl_proj, three relative-position transformer encoders, the text
// embedding, MRTE cross attention, proj), the draw z_p = m_p + noise *
// exp(logs_p) * noise_scale, and the reverse ResidualCouplingBlock
// (flow.hpp: 4 x [Flip, mean-only coupling layer around a WaveNet]).  Its
// output z is the generator's input (gsvk_decoder_*).
//
// Activations are channels-last rows [T][C] fp32 (the transpose of the
// reference's channel-major Tensor2D), with an fp16 copy wherever a
// convolution reads them.  Every Conv1d is gsvk_conv1d_f16 — fp16
// activations and weights, fp32 accumulation on the tensor cores, the
// reference's accelerated conv path (conv1d.hpp:117-150) — with the bias,
// ReLU and residual add in its epilogue.  Attention runs in fp32 on CUDA
// cores, as the reference runs it through sgemm (mha.hpp:80-113).
//
// The Flip between coupling layers is never materialised.  The flow state
// lives in two half buffers P0, P1 [T][C/2]; with orientation (a, r) the
// logical state is x = [rev^r(P_a), rev^r(P_(1-a))], so a flip is
// (a, r) -> (1 - a, !r).  Each coupling layer's pre conv reads P_a through
// input columns permuted by rev^r, and its post conv writes P_(1-a) through
// output rows permuted the same way, with weights and bias negated so that
// the epilogue's residual add (acc + bias) + x1 is the reference's x1 -= m
// exactly.  Four flips bring the orientation back to (0, 0).
#include <cmath>
#include <map>
#include <string>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_sovits_latent;

namespace gsvk {
namespace {

constexpr int kAttRows = 8;    // query rows per CTA (one warp each)
constexpr int kAttTile = 64;   // keys per shared-memory tile
constexpr int kMaxFrames = 4096;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only), zero-
// filling the destination when `valid` is false (the source is then not
// read).
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Multi-head attention for one head and kAttRows query rows per CTA
// (mha.hpp:62-202 with an all-ones mask): scores = scale * q.k (fp32 FMA
// chain over d in order, then the scale), plus, with relative tables, scale
// * q.relk[j - i + W] for |j - i| <= W (the reference's
// _relative_position_to_absolute_position gather reduces to that index);
// softmax; out = sum_j p_j v_j in key order, then sum_r p_(i+r-W) relv[r].
// The K tiles and then the V tiles of 64 keys stream through two shared
// buffers by cp.async, the next tile in flight while the current one is
// used.  Rows of a tile are dk + 4 floats: 16-byte aligned, and a quarter
// warp's float4 reads of 8 rows fall in distinct banks.
// Shared memory: Q [8][dk] | 2 x tile [64][dk+4] | scores [8][Tk].
__global__ void __launch_bounds__(256) rel_attention_kernel(
    const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk,
    const float* __restrict__ v, int ldv, int Tq, int Tk, int dk, float scale,
    const float* __restrict__ relk, const float* __restrict__ relv, int window,
    uint16_t* __restrict__ out, int ldo) {
  extern __shared__ float4 sm4[];
  float* sm = reinterpret_cast<float*>(sm4);
  const int h = blockIdx.y, i0 = blockIdx.x * kAttRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ldt = dk + 4, dk4 = dk >> 2;
  float* Qs = sm;
  float* buf0 = Qs + kAttRows * dk;  // two tiles, kAttTile * ldt floats apart
  float* S = buf0 + 2 * kAttTile * ldt;
  const int nt = (Tk + kAttTile - 1) / kAttTile;
  // tile t < nt: keys of K; nt <= t < 2 nt: values of V
  auto issue = [&](int t) {
    const bool isk = t < nt;
    const float* src = isk ? k : v;
    const int ld = isk ? ldk : ldv, j0 = (isk ? t : t - nt) * kAttTile;
    float* dst = buf0 + (t & 1) * kAttTile * ldt;
    for (int e = threadIdx.x; e < kAttTile * dk4; e += blockDim.x) {
      const int jj = e / dk4, c = e - jj * dk4, j = j0 + jj;
      const bool ok = j < Tk;
      cp_async16(dst + jj * ldt + 4 * c,
                 src + static_cast<size_t>(ok ? j : 0) * ld + h * dk + 4 * c, ok);
    }
    cp_async_commit();
  };
  issue(0);
  for (int e = threadIdx.x; e < kAttRows * dk; e += blockDim.x) {
    const int r = e / dk, d = e - r * dk, i = i0 + r;
    Qs[e] = i < Tq ? q[static_cast<size_t>(i) * ldq + h * dk + d] : 0.f;
  }
  const int i = i0 + warp;
  const bool live = i < Tq;
  float* Sr = S + static_cast<size_t>(warp) * Tk;
  const float4* Q4 = reinterpret_cast<const float4*>(Qs + warp * dk);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int nd = dk >> 5;
  for (int t = 0; t < 2 * nt; ++t) {
    if (t + 1 < 2 * nt) {
      issue(t + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* tile = buf0 + (t & 1) * kAttTile * ldt;
    if (t < nt) {
      // scores of keys j0 + lane and j0 + lane + 32
      const int j0 = t * kAttTile;
      if (live) {
        const float4* ka = reinterpret_cast<const float4*>(tile + lane * ldt);
        const float4* kb = reinterpret_cast<const float4*>(tile + (lane + 32) * ldt);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
        for (int c = 0; c < dk4; ++c) {
          const float4 qv = Q4[c], x = ka[c], y = kb[c];
          a0 = fmaf(qv.x, x.x, a0);
          a0 = fmaf(qv.y, x.y, a0);
          a0 = fmaf(qv.z, x.z, a0);
          a0 = fmaf(qv.w, x.w, a0);
          a1 = fmaf(qv.x, y.x, a1);
          a1 = fmaf(qv.y, y.y, a1);
          a1 = fmaf(qv.z, y.z, a1);
          a1 = fmaf(qv.w, y.w, a1);
        }
        if (j0 + lane < Tk) Sr[j0 + lane] = scale * a0;
        if (j0 + lane + 32 < Tk) Sr[j0 + lane + 32] = scale * a1;
      }
    } else {
      if (t == nt && live) {
        __syncwarp();
        if (relk && lane <= 2 * window) {
          const int j = i + lane - window;
          if (j >= 0 && j < Tk) {
            const float4* rk = reinterpret_cast<const float4*>(relk + lane * dk);
            float a0 = 0.f;
            for (int c = 0; c < dk4; ++c) {
              const float4 qv = Q4[c], x = rk[c];
              a0 = fmaf(qv.x, x.x, a0);
              a0 = fmaf(qv.y, x.y, a0);
              a0 = fmaf(qv.z, x.z, a0);
              a0 = fmaf(qv.w, x.w, a0);
            }
            Sr[j] += scale * a0;
          }
        }
        __syncwarp();
        float mx = -INFINITY;
        for (int j = lane; j < Tk; j += 32) mx = fmaxf(mx, Sr[j]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < Tk; j += 32) {
          const float e = expf(Sr[j] - mx);
          Sr[j] = e;
          sum += e;
        }
        const float inv = 1.f / warp_sum(sum);
        for (int j = lane; j < Tk; j += 32) Sr[j] *= inv;
        __syncwarp();
      }
      if (live) {
        const int j0 = (t - nt) * kAttTile, n = min(kAttTile, Tk - j0);
        const float* vr = tile + lane;
#pragma unroll 4
        for (int jj = 0; jj < n; ++jj) {
          const float p = Sr[j0 + jj];
          if (p == 0.f) continue;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (u < nd) acc[u] = __fadd_rn(acc[u], __fmul_rn(p, vr[jj * ldt + 32 * u]));
        }
      }
    }
    __syncthreads();
  }
  if (!live) return;
  if (relv)
    for (int r = 0; r <= 2 * window; ++r) {
      const int j = i + r - window;
      if (j < 0 || j >= Tk) continue;
      const float p = Sr[j];
      if (p == 0.f) continue;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (u < nd) acc[u] = __fadd_rn(acc[u], __fmul_rn(p, relv[r * dk + lane + 32 * u]));
    }
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (u < nd) out[static_cast<size_t>(i) * ldo + h * dk + lane + 32 * u] = f2h(acc[u]);
}

// layernorm_ct (nn_ops.hpp:26-45) on channels-last rows: one warp per frame,
// mean and biased variance over C <= 512, y = (x - mu) * inv * g + b with
// every product and sum rounded separately; fp32 and fp16 outputs.
__global__ void __launch_bounds__(256) ln_rows_kernel(const float* __restrict__ x, int T, int C,
                                                      const float* __restrict__ g,
                                                      const float* __restrict__ b, float eps,
                                                      float* __restrict__ y,
                                                      uint16_t* __restrict__ y16) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= T) return;
  const float* xr = x + static_cast<size_t>(row) * C;
  float v[16];
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const int c = lane + 32 * u;
    v[u] = c < C ? xr[c] : 0.f;
    s += v[u];
  }
  const float mu = __fdiv_rn(warp_sum(s), static_cast<float>(C));
  float s2 = 0.f;
#pragma unroll
  for (int u = 0; u < 16; ++u)
    if (lane + 32 * u < C) {
      const float d = __fsub_rn(v[u], mu);
      s2 = __fadd_rn(s2, __fmul_rn(d, d));
    }
  const float var = __fdiv_rn(warp_sum(s2), static_cast<float>(C));
  const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const int c = lane + 32 * u;
    if (c >= C) continue;
    const float o = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[u], mu), inv), g[c]), b[c]);
    y[static_cast<size_t>(row) * C + c] = o;
    y16[static_cast<size_t>(row) * C + c] = f2h(o);
  }
}

// WaveNet gate (flow.hpp:75-81): acts = tanh(a + g) * sigmoid(a' + g'), a
// the first C and a' the second C channels of the in-layer output.
__global__ void wn_gate_kernel(const float* __restrict__ a, const float* __restrict__ g, int T,
                               int C, uint16_t* __restrict__ acts) {
  const long long n = static_cast<long long>(T) * C;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / C), c = static_cast<int>(e - static_cast<long long>(t) * C);
    const float* ar = a + static_cast<size_t>(t) * 2 * C;
    const float th = tanhf(__fadd_rn(ar[c], g[c]));
    const float sg = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-__fadd_rn(ar[C + c], g[C + c]))));
    acts[e] = f2h(__fmul_rn(th, sg));
  }
}

// RVQ decode and nearest x2 (quantizer.hpp:26-38, sovits_engine.hpp:57-64):
// up[t][d] = embed[codes[t / 2]][d], fp16 (the ssl_proj conv's input).
__global__ void rvq_upsample_kernel(const int64_t* __restrict__ codes, int Tq, int D,
                                    const float* __restrict__ embed, uint16_t* __restrict__ up) {
  const long long n = static_cast<long long>(Tq) * D;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / D), d = static_cast<int>(e - static_cast<long long>(t) * D);
    up[e] = f2h(embed[static_cast<size_t>(codes[t >> 1]) * D + d]);
  }
}

// text_embedding(phones) (enc_p.hpp:62-69) as rows, fp32 and fp16.
__global__ void embed_rows_kernel(const int64_t* __restrict__ ids, int T, int C,
                                  const float* __restrict__ table, float* __restrict__ y,
                                  uint16_t* __restrict__ y16) {
  const long long n = static_cast<long long>(T) * C;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / C), c = static_cast<int>(e - static_cast<long long>(t) * C);
    const float v = table[static_cast<size_t>(ids[t]) * C + c];
    y[e] = v;
    y16[e] = f2h(v);
  }
}

__global__ void add_vec_kernel(const float* __restrict__ a, const float* __restrict__ b, int n,
                               float* __restrict__ y) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = a[i] + b[i];
}

// stats [T][2C] -> m_p, logs_p (channel-major, optional) and the flow state
// z_p = m_p + noise * exp(logs_p) * scale (sovits_engine.hpp:74-79) split
// into the halves P0 = channels [0, C/2), P1 = [C/2, C).
__global__ void draw_zp_kernel(const float* __restrict__ stats, const float* __restrict__ noise,
                               float scale, int T, int C, float* __restrict__ m_p,
                               float* __restrict__ logs_p, float* __restrict__ p0,
                               float* __restrict__ p1, uint16_t* __restrict__ p0h,
                               uint16_t* __restrict__ p1h) {
  const int half = C / 2;
  const long long n = static_cast<long long>(T) * C;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / C), c = static_cast<int>(e - static_cast<long long>(t) * C);
    const float mp = stats[static_cast<size_t>(t) * 2 * C + c];
    const float lp = stats[static_cast<size_t>(t) * 2 * C + C + c];
    const size_t cm = static_cast<size_t>(c) * T + t;
    if (m_p) m_p[cm] = mp;
    if (logs_p) logs_p[cm] = lp;
    const float nz = noise ? noise[cm] : 0.f;
    const float z = __fadd_rn(mp, __fmul_rn(__fmul_rn(nz, expf(lp)), scale));
    const size_t o = static_cast<size_t>(t) * half + (c < half ? c : c - half);
    (c < half ? p0 : p1)[o] = z;
    (c < half ? p0h : p1h)[o] = f2h(z);
  }
}

// The logical flow state x = [rev^r(P_a), rev^r(P_(1-a))] -> z channel-major
// [C][T].
__global__ void halves_to_channels_kernel(const float* __restrict__ pa,
                                          const float* __restrict__ pb, int rev, int T, int C,
                                          float* __restrict__ z) {
  const int half = C / 2;
  const long long n = static_cast<long long>(T) * C;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e / T), t = static_cast<int>(e - static_cast<long long>(c) * T);
    const int cc = c < half ? c : c - half;
    z[e] = (c < half ? pa : pb)[static_cast<size_t>(t) * half + (rev ? half - 1 - cc : cc)];
  }
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

struct DConv {
  uint16_t* w = nullptr;  // packed [k][co][ci]
  float* b = nullptr;
  int co = 0, ci = 0, k = 1;
};

struct DLayer {
  DConv qkv, o, f1, f2;
  float* relk = nullptr;
  float* relv = nullptr;
  float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
};

struct DRcl {
  DConv pre, post;
  uint16_t* cond_w = nullptr;  // [2 C nl][gin]
  float* cond_b = nullptr;
  std::vector<DConv> in, res, skip;
  int a = 0, r = 0;  // orientation of the state when this layer runs
};

}  // namespace

struct gsvk_sovits_latent {
  gsvk_sovits_latent_config cfg{};
  size_t n_codebook = 0, n_symbols = 0;
  int Tq_max = 0, Tt_max = 0;
  std::vector<void*> allocs;
  float* embed = nullptr;   // codebook [n_codebook][ssl_dim]
  float* temb_w = nullptr;  // [n_symbols][hidden]
  DConv ssl_proj, c_pre, text_pre, c_post, proj, mq, mkv, mo;
  std::vector<DLayer> enc[3];  // encoder_ssl, encoder_text, encoder2
  std::vector<DRcl> rcl;
  int fa = 0, fr = 0;  // orientation of the flow state after the last layer
  // workspaces
  int64_t *codes = nullptr, *phones = nullptr;
  uint16_t *up16 = nullptr, *y16 = nullptr, *t16 = nullptr, *att16 = nullptr, *hf16 = nullptr;
  float *y = nullptr, *s = nullptr, *temb = nullptr, *qkv = nullptr;
  float *c512 = nullptr, *mqb = nullptr, *mkvb = nullptr, *bias_eff = nullptr;
  uint16_t *c512h = nullptr, *t512h = nullptr, *sum16 = nullptr;
  float* stats = nullptr;
  float *P[2] = {nullptr, nullptr};
  uint16_t* Ph[2] = {nullptr, nullptr};
  float *h = nullptr, *a = nullptr, *out = nullptr, *g = nullptr;
  uint16_t *h16 = nullptr, *acts16 = nullptr, *out16 = nullptr;
};

namespace {

class Src {
 public:
  Src(const gsvk_gsv_tensor* t, size_t n) {
    for (size_t i = 0; i < n; ++i)
      if (t[i].name) by_[t[i].name] = &t[i];
  }
  bool has(const std::string& n) const { return by_.count(n) != 0; }
  // the tensor, checked for presence, data and element count
  const gsvk_gsv_tensor* get(const std::string& n, uint64_t numel, int* rc) const {
    auto it = by_.find(n);
    if (it == by_.end() || (!it->second->f32 && !it->second->f16)) {
      *rc = fail(GSVK_ERR_INVALID, "sovits_latent_create: missing tensor %s", n.c_str());
      return nullptr;
    }
    if (numel && it->second->numel != numel) {
      *rc = fail(GSVK_ERR_INVALID, "sovits_latent_create: %s has %llu elements, expected %llu",
                 n.c_str(), (unsigned long long)it->second->numel, (unsigned long long)numel);
      return nullptr;
    }
    return it->second;
  }
  // load_tensor_f32 (sovits_types.hpp:38-48): the fp16 copy widened when
  // the file holds one, else the fp32 copy.
  std::vector<float> f32(const std::string& n, uint64_t numel, int* rc) const {
    const gsvk_gsv_tensor* t = get(n, numel, rc);
    std::vector<float> v;
    if (!t) return v;
    v.resize(t->numel);
    for (size_t i = 0; i < v.size(); ++i)
      v[i] = t->f16 ? __half2float(__ushort_as_half(t->f16[i])) : t->f32[i];
    return v;
  }
  // load_tensor_f16 (sovits_types.hpp:76-87): the fp16 copy, else the fp32
  // copy rounded once.
  std::vector<uint16_t> f16(const std::string& n, uint64_t numel, int* rc) const {
    const gsvk_gsv_tensor* t = get(n, numel, rc);
    std::vector<uint16_t> v;
    if (!t) return v;
    v.resize(t->numel);
    for (size_t i = 0; i < v.size(); ++i) {
      if (t->f16) {
        v[i] = t->f16[i];
      } else {
        const __half hv = __float2half_rn(t->f32[i]);
        v[i] = __half_as_ushort(hv);
      }
    }
    return v;
  }

 private:
  std::map<std::string, const gsvk_gsv_tensor*> by_;
};

int dev_alloc(gsvk_sovits_latent* h, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
    cudaGetLastError();
    return fail(GSVK_ERR_NOMEM, "sovits_latent_create: %zu bytes", bytes);
  }
  h->allocs.push_back(*p);
  return GSVK_OK;
}

template <typename T>
int alloc_n(gsvk_sovits_latent* h, T** p, size_t n) {
  return dev_alloc(h, reinterpret_cast<void**>(p), n * sizeof(T));
}

template <typename T>
int upload(gsvk_sovits_latent* h, T** dst, const std::vector<T>& src) {
  if (int rc = alloc_n(h, dst, src.size())) return rc;
  return check_cuda(cudaMemcpy(*dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice),
                    "sovits_latent upload");
}

// Host-side conv weights before packing: torch [co][ci][k] fp16 and bias.
struct HConv {
  std::vector<uint16_t> w;
  std::vector<float> b;
  int co = 0, ci = 0, k = 1;
};

HConv load_conv(const Src& S, const std::string& p, int co, int ci, int k, int* rc) {
  HConv c;
  c.co = co, c.ci = ci, c.k = k;
  if (*rc) return c;
  c.w = S.f16(p + ".weight", static_cast<uint64_t>(co) * ci * k, rc);
  if (!*rc) c.b = S.has(p + ".bias") ? S.f32(p + ".bias", co, rc) : std::vector<float>(co, 0.f);
  return c;
}

// Stacks convs with the same ci and k along co (the fused q|k|v projection).
HConv stack(const std::vector<HConv>& parts) {
  HConv c = parts[0];
  for (size_t i = 1; i < parts.size(); ++i) {
    c.w.insert(c.w.end(), parts[i].w.begin(), parts[i].w.end());
    c.b.insert(c.b.end(), parts[i].b.begin(), parts[i].b.end());
    c.co += parts[i].co;
  }
  return c;
}

// Rows [r0, r0 + n) of a conv (the residual / skip halves of res_skip).
HConv rows(const HConv& c, int r0, int n) {
  HConv o;
  o.co = n, o.ci = c.ci, o.k = c.k;
  const size_t per = static_cast<size_t>(c.ci) * c.k;
  o.w.assign(c.w.begin() + r0 * per, c.w.begin() + (r0 + n) * per);
  o.b.assign(c.b.begin() + r0, c.b.begin() + r0 + n);
  return o;
}

// Packs [co][ci][k] -> tap-major [k][co][ci] and uploads.
int put_conv(gsvk_sovits_latent* h, const HConv& c, DConv* d) {
  std::vector<uint16_t> p(c.w.size());
  for (int o = 0; o < c.co; ++o)
    for (int i = 0; i < c.ci; ++i)
      for (int t = 0; t < c.k; ++t)
        p[(static_cast<size_t>(t) * c.co + o) * c.ci + i] =
            c.w[(static_cast<size_t>(o) * c.ci + i) * c.k + t];
  d->co = c.co, d->ci = c.ci, d->k = c.k;
  if (int rc = upload(h, &d->w, p)) return rc;
  return upload(h, &d->b, c.b);
}

int conv(const DConv& c, const uint16_t* x, int T, float* y, uint16_t* y16, const float* res,
         int act, cudaStream_t st, const float* bias = nullptr) {
  gsvk_conv_args a{};
  a.x = x;
  a.T = static_cast<size_t>(T);
  a.ci = static_cast<size_t>(c.ci);
  a.w = c.w;
  a.co = static_cast<size_t>(c.co);
  a.k = static_cast<size_t>(c.k);
  a.dil = 1;
  a.bias = bias ? bias : c.b;
  a.residual = res;
  a.res_scale = 1.f;
  a.act = act;
  a.y = y;
  a.y_f16 = y16;
  return gsvk_conv1d_f16(&a, st);
}

size_t att_smem(int dk, int Tk) {
  return (static_cast<size_t>(kAttRows) * dk + 2 * static_cast<size_t>(kAttTile) * (dk + 4) +
          static_cast<size_t>(kAttRows) * Tk) * sizeof(float);
}

int attention(const float* q, int ldq, const float* k, int ldk,
              const float* v, int ldv, int Tq, int Tk, int heads, int dk, const float* relk,
              const float* relv, int window, uint16_t* out, int ldo, cudaStream_t st) {
  // the kernel's 16-byte copies need 16-byte rows and bases
  if (ldq % 4 || ldk % 4 || ldv % 4 || dk % 32 || dk > 128 ||
      (reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(relk) | reinterpret_cast<uintptr_t>(relv)) % 16)
    return fail(GSVK_ERR_ALIGN, "sovits attention: unaligned operands");
  const size_t smem = att_smem(dk, Tk);
  dim3 grid((Tq + kAttRows - 1) / kAttRows, heads);
  rel_attention_kernel<<<grid, 256, smem, st>>>(q, ldq, k, ldk, v, ldv, Tq, Tk, dk,
                                                1.f / std::sqrt(static_cast<float>(dk)), relk,
                                                relv, window, out, ldo);
  return check_launch("rel_attention_kernel");
}

int layer_norm(const float* x, int T, int C, const float* g, const float* b, float* y,
               uint16_t* y16, cudaStream_t st) {
  ln_rows_kernel<<<(T + 7) / 8, 256, 0, st>>>(x, T, C, g, b, 1e-5f, y, y16);
  return check_launch("ln_rows_kernel");
}

// sovits::Encoder::forward (enc_p_parts.hpp:72-90) on rows x [T][C].
int encoder_forward(gsvk_sovits_latent* h, const std::vector<DLayer>& layers, float* x,
                    uint16_t* x16, int T, cudaStream_t st) {
  const auto& c = h->cfg;
  const int C = c.hidden, dk = C / c.heads;
  int rc = GSVK_OK;
  for (const DLayer& L : layers) {
    if (!rc) rc = conv(L.qkv, x16, T, h->qkv, nullptr, nullptr, GSVK_ACT_NONE, st);
    if (!rc)
      rc = attention(h->qkv, 3 * C, h->qkv + C, 3 * C, h->qkv + 2 * C, 3 * C, T, T, c.heads,
                     dk, L.relk, L.relv, c.window, h->att16, C, st);
    if (!rc) rc = conv(L.o, h->att16, T, h->s, nullptr, x, GSVK_ACT_NONE, st);
    if (!rc) rc = layer_norm(h->s, T, C, L.g1, L.b1, x, x16, st);
    if (!rc) rc = conv(L.f1, x16, T, nullptr, h->hf16, nullptr, GSVK_ACT_RELU, st);
    if (!rc) rc = conv(L.f2, h->hf16, T, h->s, nullptr, x, GSVK_ACT_NONE, st);
    if (!rc) rc = layer_norm(h->s, T, C, L.g2, L.b2, x, x16, st);
  }
  return rc;
}

int load_encoder(gsvk_sovits_latent* h, const Src& S, const std::string& p, int nl,
                 std::vector<DLayer>* out) {
  const auto& c = h->cfg;
  const int C = c.hidden, dk = C / c.heads, table = 2 * c.window + 1;
  int rc = GSVK_OK;
  out->resize(nl);
  for (int i = 0; i < nl && !rc; ++i) {
    const std::string ix = "." + std::to_string(i), a = p + ".attn_layers" + ix;
    DLayer& L = (*out)[i];
    HConv q = load_conv(S, a + ".conv_q", C, C, 1, &rc);
    HConv k = load_conv(S, a + ".conv_k", C, C, 1, &rc);
    HConv v = load_conv(S, a + ".conv_v", C, C, 1, &rc);
    HConv o = load_conv(S, a + ".conv_o", C, C, 1, &rc);
    HConv f1 = load_conv(S, p + ".ffn_layers" + ix + ".conv_1", c.filter, C, c.kernel, &rc);
    HConv f2 = load_conv(S, p + ".ffn_layers" + ix + ".conv_2", C, c.filter, c.kernel, &rc);
    std::vector<float> rk, rv, g1, b1, g2, b2;
    if (!rc) rk = S.f32(a + ".emb_rel_k", static_cast<uint64_t>(table) * dk, &rc);
    if (!rc) rv = S.f32(a + ".emb_rel_v", static_cast<uint64_t>(table) * dk, &rc);
    if (!rc) g1 = S.f32(p + ".norm_layers_1" + ix + ".gamma", C, &rc);
    if (!rc) b1 = S.f32(p + ".norm_layers_1" + ix + ".beta", C, &rc);
    if (!rc) g2 = S.f32(p + ".norm_layers_2" + ix + ".gamma", C, &rc);
    if (!rc) b2 = S.f32(p + ".norm_layers_2" + ix + ".beta", C, &rc);
    if (!rc) rc = put_conv(h, stack({q, k, v}), &L.qkv);
    if (!rc) rc = put_conv(h, o, &L.o);
    if (!rc) rc = put_conv(h, f1, &L.f1);
    if (!rc) rc = put_conv(h, f2, &L.f2);
    if (!rc) rc = upload(h, &L.relk, rk);
    if (!rc) rc = upload(h, &L.relv, rv);
    if (!rc) rc = upload(h, &L.g1, g1);
    if (!rc) rc = upload(h, &L.b1, b1);
    if (!rc) rc = upload(h, &L.g2, g2);
    if (!rc) rc = upload(h, &L.b2, b2);
  }
  return rc;
}

int load_flow(gsvk_sovits_latent* h, const Src& S) {
  const auto& c = h->cfg;
  const int C = c.hidden, half = C / 2, nl = c.wn_layers;
  int rc = GSVK_OK;
  h->rcl.resize(c.flows);
  // reverse order f = flows-1 .. 0, each preceded by a flip
  int a = 0, r = 0;
  for (int f = c.flows - 1; f >= 0 && !rc; --f) {
    a = 1 - a;
    r = !r;
    DRcl& L = h->rcl[f];
    L.a = a;
    L.r = r;
    const std::string p = "flow.flows." + std::to_string(2 * f);
    HConv pre = load_conv(S, p + ".pre", C, half, 1, &rc);
    HConv post = load_conv(S, p + ".post", half, C, 1, &rc);
    HConv cond = load_conv(S, p + ".enc.cond_layer", 2 * C * nl, c.gin, 1, &rc);
    if (rc) break;
    if (r) {  // x0 = rev(P_a): pre reads physical column j as channel half-1-j
      HConv t = pre;
      for (int o = 0; o < C; ++o)
        for (int j = 0; j < half; ++j)
          t.w[static_cast<size_t>(o) * half + j] =
              pre.w[static_cast<size_t>(o) * half + half - 1 - j];
      pre = t;
    }
    {  // x1 -= m as (-W) h + (-b) + x1, rows in physical order
      HConv t = post;
      for (int j = 0; j < half; ++j) {
        const int src = r ? half - 1 - j : j;
        for (int i = 0; i < C; ++i)
          t.w[static_cast<size_t>(j) * C + i] = post.w[static_cast<size_t>(src) * C + i] ^ 0x8000u;
        t.b[j] = -post.b[src];
      }
      post = t;
    }
    rc = put_conv(h, pre, &L.pre);
    if (!rc) rc = put_conv(h, post, &L.post);
    if (!rc) rc = upload(h, &L.cond_w, cond.w);
    if (!rc) rc = upload(h, &L.cond_b, cond.b);
    L.in.resize(nl);
    L.res.resize(nl);
    L.skip.resize(nl);
    for (int l = 0; l < nl && !rc; ++l) {
      HConv in =
          load_conv(S, p + ".enc.in_layers." + std::to_string(l), 2 * C, C, c.wn_kernel, &rc);
      const bool last = l + 1 == nl;
      HConv rs = load_conv(S, p + ".enc.res_skip_layers." + std::to_string(l), last ? C : 2 * C,
                           C, 1, &rc);
      if (rc) break;
      rc = put_conv(h, in, &L.in[l]);
      if (!rc && !last) rc = put_conv(h, rows(rs, 0, C), &L.res[l]);
      if (!rc) rc = put_conv(h, last ? rs : rows(rs, C, C), &L.skip[l]);
    }
  }
  h->fa = a;
  h->fr = r;
  return rc;
}

int create_impl(gsvk_sovits_latent* h, const Src& S) {
  const auto& c = h->cfg;
  const int C = c.hidden, D = c.ssl_dim, MH = c.mrte_hidden, F = c.filter;
  int rc = GSVK_OK;
  // codebook and text embedding: their sizes come from the file
  std::vector<float> embed = S.f32("quantizer.vq.layers.0._codebook.embed", 0, &rc);
  if (!rc && (embed.empty() || embed.size() % D))
    rc = fail(GSVK_ERR_INVALID, "sovits_latent_create: codebook is not [n][%d]", D);
  if (!rc) h->n_codebook = embed.size() / D;
  std::vector<float> temb;
  if (!rc) temb = S.f32("enc_p.text_embedding.weight", 0, &rc);
  if (!rc && (temb.empty() || temb.size() % C))
    rc = fail(GSVK_ERR_INVALID, "sovits_latent_create: text embedding is not [n][%d]", C);
  if (!rc) h->n_symbols = temb.size() / C;
  if (!rc) rc = upload(h, &h->embed, embed);
  if (!rc) rc = upload(h, &h->temb_w, temb);
  HConv ssl = load_conv(S, "enc_p.ssl_proj", C, D, 1, &rc);
  HConv cp = load_conv(S, "enc_p.mrte.c_pre", MH, C, 1, &rc);
  HConv tp = load_conv(S, "enc_p.mrte.text_pre", MH, C, 1, &rc);
  HConv cpo = load_conv(S, "enc_p.mrte.c_post", C, MH, 1, &rc);
  HConv pj = load_conv(S, "enc_p.proj", 2 * C, C, 1, &rc);
  const std::string ca = "enc_p.mrte.cross_attention";
  HConv q = load_conv(S, ca + ".conv_q", MH, MH, 1, &rc);
  HConv k = load_conv(S, ca + ".conv_k", MH, MH, 1, &rc);
  HConv v = load_conv(S, ca + ".conv_v", MH, MH, 1, &rc);
  HConv o = load_conv(S, ca + ".conv_o", MH, MH, 1, &rc);
  if (!rc) rc = put_conv(h, ssl, &h->ssl_proj);
  if (!rc) rc = put_conv(h, cp, &h->c_pre);
  if (!rc) rc = put_conv(h, tp, &h->text_pre);
  if (!rc) rc = put_conv(h, cpo, &h->c_post);
  if (!rc) rc = put_conv(h, pj, &h->proj);
  if (!rc) rc = put_conv(h, q, &h->mq);
  if (!rc) rc = put_conv(h, stack({k, v}), &h->mkv);
  if (!rc) rc = put_conv(h, o, &h->mo);
  if (!rc) rc = load_encoder(h, S, "enc_p.encoder_ssl", c.layers_ssl, &h->enc[0]);
  if (!rc) rc = load_encoder(h, S, "enc_p.encoder_text", c.layers_text, &h->enc[1]);
  if (!rc) rc = load_encoder(h, S, "enc_p.encoder2", c.layers_2, &h->enc[2]);
  if (!rc) rc = load_flow(h, S);
  if (rc) return rc;
  // workspaces
  const size_t Tq = h->Tq_max, Tt = h->Tt_max, Tm = std::max(Tq, Tt);
  const size_t W = std::max<size_t>(C, MH);
  if (!rc) rc = alloc_n(h, &h->codes, Tq / 2);
  if (!rc) rc = alloc_n(h, &h->phones, Tt);
  if (!rc) rc = alloc_n(h, &h->up16, Tq * D);
  if (!rc) rc = alloc_n(h, &h->y, Tq * C);
  if (!rc) rc = alloc_n(h, &h->y16, Tq * C);
  if (!rc) rc = alloc_n(h, &h->s, Tm * C);
  if (!rc) rc = alloc_n(h, &h->temb, Tt * C);
  if (!rc) rc = alloc_n(h, &h->t16, Tt * C);
  if (!rc) rc = alloc_n(h, &h->qkv, Tm * 3 * C);
  if (!rc) rc = alloc_n(h, &h->att16, Tm * W);
  if (!rc) rc = alloc_n(h, &h->hf16, Tm * F);
  if (!rc) rc = alloc_n(h, &h->c512, Tq * MH);
  if (!rc) rc = alloc_n(h, &h->c512h, Tq * MH);
  if (!rc) rc = alloc_n(h, &h->t512h, Tt * MH);
  if (!rc) rc = alloc_n(h, &h->mqb, Tq * MH);
  if (!rc) rc = alloc_n(h, &h->mkvb, Tt * 2 * MH);
  if (!rc) rc = alloc_n(h, &h->sum16, Tq * MH);
  if (!rc) rc = alloc_n(h, &h->bias_eff, MH);
  if (!rc) rc = alloc_n(h, &h->stats, Tq * 2 * C);
  for (int i = 0; i < 2 && !rc; ++i) {
    rc = alloc_n(h, &h->P[i], Tq * C / 2);
    if (!rc) rc = alloc_n(h, &h->Ph[i], Tq * C / 2);
  }
  if (!rc) rc = alloc_n(h, &h->h, Tq * C);
  if (!rc) rc = alloc_n(h, &h->h16, Tq * C);
  if (!rc) rc = alloc_n(h, &h->a, Tq * 2 * C);
  if (!rc) rc = alloc_n(h, &h->acts16, Tq * C);
  if (!rc) rc = alloc_n(h, &h->out, Tq * C);
  if (!rc) rc = alloc_n(h, &h->out16, Tq * C);
  if (!rc) rc = alloc_n(h, &h->g, static_cast<size_t>(c.flows) * 2 * C * c.wn_layers);
  if (!rc)  // the envelope's largest launch (dk 128, kMaxFrames keys), so that
            // engines of different sizes never lower each other's limit
    rc = check_cuda(cudaFuncSetAttribute(rel_attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(att_smem(128, kMaxFrames))),
                    "cudaFuncSetAttribute(rel_attention_kernel)");
  return rc;
}

}  // namespace

extern "C" {

int gsvk_sovits_latent_destroy(gsvk_sovits_latent_t h) {
  if (!h) return GSVK_OK;
  for (void* p : h->allocs) cudaFree(p);
  delete h;
  return GSVK_OK;
}

int gsvk_sovits_latent_create(const gsvk_sovits_latent_config* cfg, const gsvk_gsv_tensor* tensors,
                              size_t n, gsvk_sovits_latent_t* out) {
  if (!cfg || !tensors || !out)
    return fail(GSVK_ERR_INVALID, "sovits_latent_create: null argument");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  const auto& c = *cfg;
  const bool ok =
      c.hidden > 0 && c.hidden % 16 == 0 && c.hidden <= 512 && c.heads > 0 &&
      c.hidden % c.heads == 0 && (c.hidden / c.heads) % 32 == 0 && c.hidden / c.heads <= 128 &&
      c.mrte_hidden > 0 && c.mrte_hidden % 8 == 0 && c.mrte_heads > 0 &&
      c.mrte_hidden % c.mrte_heads == 0 && (c.mrte_hidden / c.mrte_heads) % 32 == 0 &&
      c.mrte_hidden / c.mrte_heads <= 128 && c.ssl_dim > 0 && c.ssl_dim % 8 == 0 &&
      c.filter > 0 && c.filter % 8 == 0 && c.kernel > 0 && c.kernel % 2 == 1 &&
      c.window >= 0 && 2 * c.window + 1 <= 32 && c.layers_ssl >= 0 && c.layers_text >= 0 &&
      c.layers_2 >= 0 && c.gin > 0 && c.flows > 0 && c.wn_layers > 0 && c.wn_kernel > 0 &&
      c.wn_kernel % 2 == 1 && c.max_codes > 0 && c.max_phones > 0 &&
      2 * c.max_codes <= static_cast<size_t>(kMaxFrames) &&
      c.max_phones <= static_cast<size_t>(kMaxFrames);
  if (!ok)
    return fail(GSVK_ERR_INVALID,
                "sovits_latent_create: configuration outside the supported envelope");
  auto* h = new gsvk_sovits_latent();
  h->cfg = c;
  h->Tq_max = static_cast<int>(2 * c.max_codes);
  h->Tt_max = static_cast<int>(c.max_phones);
  const Src S(tensors, n);
  if (int rc = create_impl(h, S)) {
    gsvk_sovits_latent_destroy(h);
    return rc;
  }
  *out = h;
  return GSVK_OK;
}

int gsvk_sovits_latent_create_from_gsv(gsvk_gsv_t f, const gsvk_sovits_latent_config* cfg,
                                       gsvk_sovits_latent_t* out) {
  if (!f || !out) return fail(GSVK_ERR_INVALID, "sovits_latent_create_from_gsv: null argument");
  const size_t n = gsvk_gsv_count(f);
  std::vector<gsvk_gsv_tensor> t(n);
  for (size_t i = 0; i < n; ++i)
    if (int rc = gsvk_gsv_tensor_at(f, i, &t[i])) return rc;
  return gsvk_sovits_latent_create(cfg, t.data(), n, out);
}

int gsvk_sovits_latent_forward(gsvk_sovits_latent_t h, const int64_t* codes, size_t n_codes,
                               const int64_t* phones, size_t n_phones, const float* ge,
                               const float* ge_text, const float* noise, float* z, float* m_p,
                               float* logs_p, gsvk_stream_t stream) {
  if (!h || !codes || !phones || !ge || !ge_text || !z)
    return fail(GSVK_ERR_INVALID, "sovits_latent_forward: null argument");
  if (n_codes == 0 || n_phones == 0 || n_codes > h->cfg.max_codes || n_phones > h->cfg.max_phones)
    return fail(GSVK_ERR_INVALID,
                "sovits_latent_forward: %zu codes / %zu phones outside 1..%zu / 1..%zu",
                n_codes, n_phones, h->cfg.max_codes, h->cfg.max_phones);
  for (size_t i = 0; i < n_codes; ++i)  // quantizer.hpp:30-31
    if (codes[i] < 0 || static_cast<size_t>(codes[i]) >= h->n_codebook)
      return fail(GSVK_ERR_INVALID, "sovits_latent_forward: code index out of range at %zu", i);
  for (size_t i = 0; i < n_phones; ++i)  // enc_p.hpp:64-65
    if (phones[i] < 0 || static_cast<size_t>(phones[i]) >= h->n_symbols)
      return fail(GSVK_ERR_INVALID, "sovits_latent_forward: phone id out of range at %zu", i);
  const auto& c = h->cfg;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int Tq = static_cast<int>(2 * n_codes), Tt = static_cast<int>(n_phones);
  const int C = c.hidden, D = c.ssl_dim, MH = c.mrte_hidden, nl = c.wn_layers;
  int rc = check_cuda(cudaMemcpyAsync(h->codes, codes, n_codes * 8, cudaMemcpyHostToDevice, st),
                      "sovits_latent codes");
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(h->phones, phones, n_phones * 8, cudaMemcpyHostToDevice, st),
                    "sovits_latent phones");
  if (rc) return rc;
  // 1-2. codes -> [Tq][ssl_dim] fp16
  rvq_upsample_kernel<<<grid_for(static_cast<long long>(Tq) * D), 256, 0, st>>>(h->codes, Tq, D,
                                                                              h->embed, h->up16);
  if ((rc = check_launch("rvq_upsample_kernel"))) return rc;
  // 3. TextEncoder (enc_p.hpp:45-91)
  rc = conv(h->ssl_proj, h->up16, Tq, h->y, h->y16, nullptr, GSVK_ACT_NONE, st);
  if (!rc) rc = encoder_forward(h, h->enc[0], h->y, h->y16, Tq, st);
  if (!rc) {
    embed_rows_kernel<<<grid_for(static_cast<long long>(Tt) * C), 256, 0, st>>>(
        h->phones, Tt, C, h->temb_w, h->temb, h->t16);
    rc = check_launch("embed_rows_kernel");
  }
  if (!rc) rc = encoder_forward(h, h->enc[1], h->temb, h->t16, Tt, st);
  // MRTE (enc_p_parts.hpp:111-129): c_post(attn(c_pre y, text_pre t) + c_pre y + ge_text)
  if (!rc) rc = conv(h->c_pre, h->y16, Tq, h->c512, h->c512h, nullptr, GSVK_ACT_NONE, st);
  if (!rc) rc = conv(h->text_pre, h->t16, Tt, nullptr, h->t512h, nullptr, GSVK_ACT_NONE, st);
  if (!rc) rc = conv(h->mq, h->c512h, Tq, h->mqb, nullptr, nullptr, GSVK_ACT_NONE, st);
  if (!rc) rc = conv(h->mkv, h->t512h, Tt, h->mkvb, nullptr, nullptr, GSVK_ACT_NONE, st);
  if (!rc)
    rc = attention(h->mqb, MH, h->mkvb, 2 * MH, h->mkvb + MH, 2 * MH, Tq, Tt, c.mrte_heads,
                   MH / c.mrte_heads, nullptr, nullptr, 0, h->att16, MH, st);
  if (!rc) {
    add_vec_kernel<<<(MH + 255) / 256, 256, 0, st>>>(h->mo.b, ge_text, MH, h->bias_eff);
    rc = check_launch("add_vec_kernel");
  }
  if (!rc)
    rc = conv(h->mo, h->att16, Tq, nullptr, h->sum16, h->c512, GSVK_ACT_NONE, st, h->bias_eff);
  if (!rc) rc = conv(h->c_post, h->sum16, Tq, h->y, h->y16, nullptr, GSVK_ACT_NONE, st);
  if (!rc) rc = encoder_forward(h, h->enc[2], h->y, h->y16, Tq, st);
  if (!rc) rc = conv(h->proj, h->y16, Tq, h->stats, nullptr, nullptr, GSVK_ACT_NONE, st);
  // 4. z_p
  if (!rc) {
    draw_zp_kernel<<<grid_for(static_cast<long long>(Tq) * C), 256, 0, st>>>(
        h->stats, noise, c.noise_scale, Tq, C, m_p, logs_p, h->P[0], h->P[1], h->Ph[0], h->Ph[1]);
    rc = check_launch("draw_zp_kernel");
  }
  // 5. reverse flow: the cond vectors (one frame, fp32 input), then the layers
  for (int f = 0; f < c.flows && !rc; ++f)
    rc = gemv_ex(h->rcl[f].cond_w, ge, 0, h->g + static_cast<size_t>(f) * 2 * C * nl, nullptr,
                 static_cast<size_t>(2 * C * nl), static_cast<size_t>(c.gin), h->rcl[f].cond_b,
                 nullptr, GSVK_ACT_NONE, 0.f, st);
  for (int f = c.flows - 1; f >= 0 && !rc; --f) {
    const DRcl& L = h->rcl[f];
    const float* g = h->g + static_cast<size_t>(f) * 2 * C * nl;
    rc = conv(L.pre, h->Ph[L.a], Tq, h->h, h->h16, nullptr, GSVK_ACT_NONE, st);
    for (int l = 0; l < nl && !rc; ++l) {
      const bool last = l + 1 == nl;
      rc = conv(L.in[l], h->h16, Tq, h->a, nullptr, nullptr, GSVK_ACT_NONE, st);
      if (!rc) {
        wn_gate_kernel<<<grid_for(static_cast<long long>(Tq) * C), 256, 0, st>>>(
            h->a, g + static_cast<size_t>(l) * 2 * C, Tq, C, h->acts16);
        rc = check_launch("wn_gate_kernel");
      }
      if (!rc && !last) rc = conv(L.res[l], h->acts16, Tq, h->h, h->h16, h->h, GSVK_ACT_NONE, st);
      if (!rc)
        rc = conv(L.skip[l], h->acts16, Tq, h->out, last ? h->out16 : nullptr,
                  l ? h->out : nullptr, GSVK_ACT_NONE, st);
    }
    if (!rc) rc = conv(L.post, h->out16, Tq, h->P[1 - L.a], h->Ph[1 - L.a], h->P[1 - L.a],
                       GSVK_ACT_NONE, st);
  }
  if (!rc) {
    halves_to_channels_kernel<<<grid_for(static_cast<long long>(Tq) * C), 256, 0, st>>>(
        h->P[h->fa], h->P[1 - h->fa], h->fr, Tq, C, z);
    rc = check_launch("halves_to_channels_kernel");
  }
  return rc;
}

}  // extern "C"
