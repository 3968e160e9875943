// conv.cu — SoVITS convolutions as implicit GEMMs on the tensor-core kernel
// (gemm_tc.cuh) and the HiFi-GAN generator (dec.hpp:265-345) built from them.
//
// Activations are channels-last ([T, C], channels contiguous, fp16 operands,
// fp32 residual stream) so that a conv tap is a row shift of the A operand:
// TMA fetches rows t + tap*dil - pad of x[T, Ci] and zero-fills rows outside
// [0, T), which is exactly the reference's same padding (conv1d.hpp:165-176)
// without an im2col buffer.  Weights are packed once at load into
// [k][Co][Ci] (tap-major, the reference ConvT phase layout conv1d.hpp:226-232),
// so tap t of the B operand is rows t*Co .. t*Co+Co-1.
//
// ConvTranspose1d (conv1d.hpp:250-359) runs polyphase: output phase r takes
// the taps j = r + m*u and writes rows q*u + r - pad directly, so there is no
// scatter-add and no atomics.
//
// Rounding points follow the reference's accelerated path: every conv input
// is rounded to fp16 (im2col_to_panel_f16, sovits_types.hpp:178), the
// residual stream and the resblock mean stay fp32 (dec.hpp:303-335).
#include <algorithm>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_decoder;

namespace gsvk {

namespace {

// torch Conv1d [Co, Ci, k] -> [k][Co][Ci]
__global__ void pack_conv_kernel(const uint16_t* __restrict__ w, int Co, int Ci, int k,
                                 uint16_t* __restrict__ out) {
  const size_t n = static_cast<size_t>(Co) * Ci * k;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int ci = static_cast<int>(i % Ci);
    const size_t r = i / Ci;
    const int co = static_cast<int>(r % Co), t = static_cast<int>(r / Co);
    out[i] = w[(static_cast<size_t>(co) * Ci + ci) * k + t];
  }
}

// torch ConvTranspose1d [Ci, Co, k] -> [k][Co][Ci]
__global__ void pack_convt_kernel(const uint16_t* __restrict__ w, int Ci, int Co, int k,
                                  uint16_t* __restrict__ out) {
  const size_t n = static_cast<size_t>(Co) * Ci * k;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int ci = static_cast<int>(i % Ci);
    const size_t r = i / Ci;
    const int co = static_cast<int>(r % Co), t = static_cast<int>(r / Co);
    out[i] = w[(static_cast<size_t>(ci) * Co + co) * k + t];
  }
}

// channel-major fp32 [C, T] -> channels-last fp16 [T, C] (32 x 32 tiles)
__global__ void cm_to_cl16_kernel(const float* __restrict__ x, int C, int T,
                                  uint16_t* __restrict__ y) {
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && t < T) ? x[static_cast<size_t>(c) * T + t] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    if (t < T && c < C) y[static_cast<size_t>(t) * C + c] = f2h(tile[threadIdx.x][i]);
  }
}

// channels-last fp32 [T, C] -> channel-major fp32 [C, T]
__global__ void cl_to_cm32_kernel(const float* __restrict__ x, int T, int C, float* __restrict__ y) {
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int t = t0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && t < T) ? x[static_cast<size_t>(t) * C + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, t = t0 + threadIdx.x;
    if (t < T && c < C) y[static_cast<size_t>(c) * T + t] = tile[threadIdx.x][i];
  }
}

// Resblock mean (dec.hpp:323-334): j == 0: sum = cur * (1/3); else
// sum = sum + cur * (1/3) (separately rounded multiply and add); after the
// last resblock also emit the next stage's fp16 input lrelu(sum, slope).
unsigned grid_for(size_t n) {
  size_t g = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(sm_count()) * 16;
  return static_cast<unsigned>(std::max<size_t>(1, std::min(g, cap)));
}

TcEpilogue conv_epilogue(const gsvk_conv_args* c) {
  TcEpilogue e = make_epilogue();
  e.bias = c->bias;
  e.residual = c->residual;
  e.res_scale = c->residual ? c->res_scale : 1.f;
  e.c32 = c->y;
  e.c16 = c->y_f16;
  e.c16_act = c->y_f16_act;
  e.ld_c32 = e.ld_c16 = e.ld_res = e.ld_c16_act = static_cast<long long>(c->co);
  e.act = c->act;
  e.slope = c->slope;
  e.act2 = c->act2;
  e.slope2 = c->slope2;
  return e;
}

int check_conv(const gsvk_conv_args* c, const char* who, bool other_out) {
  if (!c || !c->x || !c->w || (!c->y && !c->y_f16 && !c->y_f16_act && !other_out) || c->T == 0 ||
      c->ci == 0 || c->co == 0 || c->k == 0 || c->dil == 0)
    return fail(GSVK_ERR_INVALID, "%s: null pointer or zero size", who);
  if (c->T > 0x3fffffff || c->ci > 65536 || c->co > 65536 || c->k > 64 || c->dil > 4096)
    return fail(GSVK_ERR_UNSUPPORTED, "%s: size outside the kernel envelope", who);
  if (c->ci % 8 != 0)
    return fail(GSVK_ERR_ALIGN, "%s: input channels must be a multiple of 8 (16-byte rows)", who);
  const int a = c->act, a2 = c->act2;
  if (a < GSVK_ACT_NONE || a > GSVK_ACT_TANH || a2 < GSVK_ACT_NONE || a2 > GSVK_ACT_TANH)
    return fail(GSVK_ERR_INVALID, "%s: bad activation", who);
  return GSVK_OK;
}

}  // namespace

// ConvT phase r: rows q in [q0, qmax] produce output rows q*u + r - pad.
static void convt_phase_rows(long long T, int u, int pad, int r, long long* q0, long long* qmax) {
  const long long num = pad - r;
  *q0 = num > 0 ? (num + u - 1) / u : 0;
  const long long top = T * u - 1 + pad - r;
  *qmax = top >= 0 ? top / u : -1;
}

// Engine-internal additions to a conv launch (not part of gsvk_conv_args).
struct ConvFuse {
  float* mean_sum = nullptr;  // TcEpilogue running mean
  float mean_scale = 1.f;
  int mean_first = 0;
  int pdl = 0;                // TcProblem::pdl (the weights are immutable)
};

static void apply_fuse(const ConvFuse* f, TcProblem* p, TcEpilogue* e) {
  if (!f) return;
  e->mean_sum = f->mean_sum;
  e->mean_scale = f->mean_scale;
  e->mean_first = f->mean_first;
  p->pdl = f->pdl;
}

int conv1d_run(const gsvk_conv_args* c, cudaStream_t st, const ConvFuse* f = nullptr) {
  if (int rc = check_conv(c, "conv1d", f && f->mean_sum)) return rc;
  const long long dil = static_cast<long long>(c->dil), k = static_cast<long long>(c->k);
  TcProblem p{};
  p.M = static_cast<int>(c->T);
  p.N = static_cast<int>(c->co);
  p.kc = static_cast<int>(c->ci);
  p.taps = static_cast<int>(k);
  p.dil = static_cast<int>(dil);
  p.pad = static_cast<int>((k - 1) * dil / 2);  // conv1d.hpp:165 same padding
  p.b_tap_rows = static_cast<int>(c->co);
  p.convt = 0;
  p.phases = 1;
  p.out_rows = static_cast<int>(c->T);
  TcEpilogue e = conv_epilogue(c);
  apply_fuse(f, &p, &e);
  return tc_run(c->x, (long long)c->T, (long long)c->ci, c->w, k * (long long)c->co,
                (long long)c->ci, p, e, 0, st);
}

int convt1d_run(const gsvk_conv_args* c, cudaStream_t st, const ConvFuse* f = nullptr) {
  if (int rc = check_conv(c, "convt1d", f && f->mean_sum)) return rc;
  const int u = static_cast<int>(c->dil), k = static_cast<int>(c->k);
  if (k < u || (k - u) % 2 != 0)
    return fail(GSVK_ERR_UNSUPPORTED, "convt1d: needs kernel >= stride and (kernel - stride) even");
  const int pad = (k - u) / 2;  // conv1d.hpp:263
  long long mrows = 0;
  for (int r = 0; r < u; ++r) {
    long long q0, qmax;
    convt_phase_rows(static_cast<long long>(c->T), u, pad, r, &q0, &qmax);
    mrows = std::max(mrows, qmax - q0 + 1);
  }
  TcProblem p{};
  p.M = static_cast<int>(mrows);
  p.N = static_cast<int>(c->co);
  p.kc = static_cast<int>(c->ci);
  p.taps = k;
  p.dil = u;
  p.pad = pad;
  p.b_tap_rows = static_cast<int>(c->co);
  p.convt = 1;
  p.phases = u;
  p.out_rows = static_cast<int>(c->T * u);
  TcEpilogue e = conv_epilogue(c);
  apply_fuse(f, &p, &e);
  return tc_run(c->x, (long long)c->T, (long long)c->ci, c->w, (long long)k * (long long)c->co,
                (long long)c->ci, p, e, 0, st);
}

// ---------------------------------------------------------------- generator
struct DecoderEngine {
  gsvk_decoder_config cfg{};
  int n_convs = 0;
  std::vector<uint16_t*> w;  // packed [k][Co][Ci]
  std::vector<float*> b;     // [Co] or null
  std::vector<int> ci, co, kk;
  void* wmem = nullptr;
  void* amem = nullptr;
  size_t max_frames = 0, max_elems = 0;
  uint16_t *in16 = nullptr, *a16 = nullptr, *xu16 = nullptr, *t16a = nullptr, *t16b = nullptr;
  float *xu32 = nullptr, *cur32 = nullptr, *sum32 = nullptr, *wav_cl = nullptr;
  int launches = 0;
  // The layers between conv_pre and conv_post touch only the buffers above,
  // so they are captured once per input length into a CUDA graph (on a
  // private stream) and replayed on the caller's stream.
  struct Graph {
    size_t T;
    cudaGraphExec_t exec;
    int launches;
    unsigned long long used;
  };
  static constexpr size_t kMaxGraphs = 8;
  bool use_graph = true;
  cudaStream_t capture = nullptr;
  std::vector<Graph> graphs;
  unsigned long long tick = 0;
};

}  // namespace gsvk

using namespace gsvk;

struct gsvk_decoder : gsvk::DecoderEngine {};

extern "C" {

int gsvk_conv1d_pack_weight(const uint16_t* w_torch, size_t co, size_t ci, size_t k,
                            uint16_t* packed, gsvk_stream_t stream) {
  if (!w_torch || !packed || !co || !ci || !k) return fail(GSVK_ERR_INVALID, "conv pack: null");
  pack_conv_kernel<<<grid_for(co * ci * k), 256, 0, as_cuda(stream)>>>(w_torch, (int)co, (int)ci,
                                                                       (int)k, packed);
  return check_launch("pack_conv_kernel");
}

int gsvk_convt1d_pack_weight(const uint16_t* w_torch, size_t ci, size_t co, size_t k,
                             uint16_t* packed, gsvk_stream_t stream) {
  if (!w_torch || !packed || !co || !ci || !k) return fail(GSVK_ERR_INVALID, "convt pack: null");
  pack_convt_kernel<<<grid_for(co * ci * k), 256, 0, as_cuda(stream)>>>(w_torch, (int)ci, (int)co,
                                                                        (int)k, packed);
  return check_launch("pack_convt_kernel");
}

int gsvk_channels_to_rows_f16(const float* x, size_t C, size_t T, uint16_t* y,
                              gsvk_stream_t stream) {
  if (!x || !y || !C || !T) return fail(GSVK_ERR_INVALID, "channels_to_rows: null or empty");
  dim3 grid((unsigned)((T + 31) / 32), (unsigned)((C + 31) / 32));
  cm_to_cl16_kernel<<<grid, dim3(32, 8), 0, as_cuda(stream)>>>(x, (int)C, (int)T, y);
  return check_launch("cm_to_cl16_kernel");
}

int gsvk_rows_to_channels_f32(const float* x, size_t T, size_t C, float* y, gsvk_stream_t stream) {
  if (!x || !y || !C || !T) return fail(GSVK_ERR_INVALID, "rows_to_channels: null or empty");
  dim3 grid((unsigned)((T + 31) / 32), (unsigned)((C + 31) / 32));
  cl_to_cm32_kernel<<<grid, dim3(32, 8), 0, as_cuda(stream)>>>(x, (int)T, (int)C, y);
  return check_launch("cl_to_cm32_kernel");
}

int gsvk_conv1d_f16(const gsvk_conv_args* args, gsvk_stream_t stream) {
  return conv1d_run(args, as_cuda(stream));
}

int gsvk_convt1d_f16(const gsvk_conv_args* args, gsvk_stream_t stream) {
  return convt1d_run(args, as_cuda(stream));
}

size_t gsvk_decoder_out_len(const gsvk_decoder_config* cfg, size_t T) {
  if (!cfg) return 0;
  size_t t = T;
  for (int s = 0; s < cfg->n_stages; ++s) t *= (size_t)cfg->up_rate[s];
  return t;
}

int gsvk_decoder_destroy(gsvk_decoder_t h) {
  if (!h) return GSVK_OK;
  if (!h->graphs.empty()) cudaDeviceSynchronize();  // no replay may be in flight
  for (auto& g : h->graphs) cudaGraphExecDestroy(g.exec);
  if (h->capture) cudaStreamDestroy(h->capture);
  if (h->wmem) cudaFree(h->wmem);
  if (h->amem) cudaFree(h->amem);
  delete h;
  return GSVK_OK;
}

int gsvk_decoder_create(const gsvk_decoder_config* cfg, const uint16_t* const* w_host,
                        const float* const* b_host, gsvk_decoder_t* out) {
  if (!cfg || !w_host || !b_host || !out) return fail(GSVK_ERR_INVALID, "decoder_create: null");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  if (cfg->n_stages < 1 || cfg->n_stages > 8 || cfg->in_ch <= 0 || cfg->ch0 <= 0 ||
      cfg->max_frames <= 0 || cfg->in_ch % 8 || cfg->conv_pre_k <= 0 || cfg->conv_post_k <= 0)
    return fail(GSVK_ERR_INVALID, "decoder_create: bad configuration");
  auto* e = new gsvk_decoder();
  e->cfg = *cfg;
  // shapes of every conv in the oracle/weights order
  int C = cfg->ch0;
  auto add = [&](int ci, int co, int k) {
    e->ci.push_back(ci);
    e->co.push_back(co);
    e->kk.push_back(k);
  };
  add(cfg->in_ch, C, cfg->conv_pre_k);
  for (int s = 0; s < cfg->n_stages; ++s) {
    const int Cn = C / 2;
    if (Cn % 8 != 0 || C % 8 != 0) {
      delete e;
      return fail(GSVK_ERR_UNSUPPORTED, "decoder_create: channels must stay multiples of 8");
    }
    add(C, Cn, cfg->up_k[s]);
    for (int j = 0; j < 3; ++j)
      for (int p = 0; p < 3; ++p) {
        add(Cn, Cn, cfg->res_k[j]);
        add(Cn, Cn, cfg->res_k[j]);
      }
    C = Cn;
  }
  add(C, 1, cfg->conv_post_k);
  e->n_convs = (int)e->ci.size();
  // weights: packed fp16 + fp32 bias (one allocation) + staging for the torch layout
  size_t off = 0, stage_elems = 0;
  std::vector<size_t> woff(e->n_convs), boff(e->n_convs);
  for (int i = 0; i < e->n_convs; ++i) {
    const size_t n = (size_t)e->ci[i] * e->co[i] * e->kk[i];
    woff[i] = off;
    off += (n * 2 + 255) / 256 * 256;
    boff[i] = off;
    off += ((size_t)e->co[i] * 4 + 255) / 256 * 256;
    stage_elems = std::max(stage_elems, n);
  }
  const size_t stage_off = off;
  off += stage_elems * 2;
  if (cudaMalloc(&e->wmem, off) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return fail(GSVK_ERR_NOMEM, "decoder_create: weights");
  }
  uint8_t* base = static_cast<uint8_t*>(e->wmem);
  uint16_t* stage = reinterpret_cast<uint16_t*>(base + stage_off);
  for (int i = 0; i < e->n_convs; ++i) {
    const size_t n = (size_t)e->ci[i] * e->co[i] * e->kk[i];
    uint16_t* wp = reinterpret_cast<uint16_t*>(base + woff[i]);
    float* bp = reinterpret_cast<float*>(base + boff[i]);
    int rc = check_cuda(cudaMemcpy(stage, w_host[i], n * 2, cudaMemcpyHostToDevice), "upload w");
    if (rc) { gsvk_decoder_destroy(e); return rc; }
    const bool is_convt = (i > 0 && i < e->n_convs - 1 && (i - 1) % 19 == 0);
    rc = is_convt ? gsvk_convt1d_pack_weight(stage, e->ci[i], e->co[i], e->kk[i], wp, nullptr)
                  : gsvk_conv1d_pack_weight(stage, e->co[i], e->ci[i], e->kk[i], wp, nullptr);
    if (rc) { gsvk_decoder_destroy(e); return rc; }
    if (b_host[i]) {
      rc = check_cuda(cudaMemcpy(bp, b_host[i], (size_t)e->co[i] * 4, cudaMemcpyHostToDevice),
                      "upload b");
      if (rc) { gsvk_decoder_destroy(e); return rc; }
      e->b.push_back(bp);
    } else {
      e->b.push_back(nullptr);
    }
    e->w.push_back(wp);
  }
  if (int rc = check_cuda(cudaDeviceSynchronize(), "decoder pack")) {
    gsvk_decoder_destroy(e);
    return rc;
  }
  // activations for max_frames input frames
  e->max_frames = (size_t)cfg->max_frames;
  size_t t = e->max_frames, maxe = t * (size_t)cfg->ch0;
  C = cfg->ch0;
  for (int s = 0; s < cfg->n_stages; ++s) {
    t *= (size_t)cfg->up_rate[s];
    C /= 2;
    maxe = std::max(maxe, t * (size_t)C);
  }
  e->max_elems = maxe;
  const size_t n16 = (maxe * 2 + 255) / 256 * 256, n32 = (maxe * 4 + 255) / 256 * 256;
  const size_t in_bytes = (e->max_frames * cfg->in_ch * 2 + 255) / 256 * 256;
  const size_t wav_bytes = (t * 4 + 255) / 256 * 256;
  if (cudaMalloc(&e->amem, in_bytes + 4 * n16 + 3 * n32 + wav_bytes) != cudaSuccess) {
    cudaGetLastError();
    gsvk_decoder_destroy(e);
    return fail(GSVK_ERR_NOMEM, "decoder_create: activations");
  }
  uint8_t* a = static_cast<uint8_t*>(e->amem);
  e->in16 = reinterpret_cast<uint16_t*>(a);
  a += in_bytes;
  e->a16 = reinterpret_cast<uint16_t*>(a);
  e->xu16 = reinterpret_cast<uint16_t*>(a + n16);
  e->t16a = reinterpret_cast<uint16_t*>(a + 2 * n16);
  e->t16b = reinterpret_cast<uint16_t*>(a + 3 * n16);
  a += 4 * n16;
  e->xu32 = reinterpret_cast<float*>(a);
  e->cur32 = reinterpret_cast<float*>(a + n32);
  e->sum32 = reinterpret_cast<float*>(a + 2 * n32);
  e->wav_cl = reinterpret_cast<float*>(a + 3 * n32);
  if (int rc = check_cuda(cudaStreamCreateWithFlags(&e->capture, cudaStreamNonBlocking),
                          "decoder capture stream")) {
    gsvk_decoder_destroy(e);
    return rc;
  }
  *out = e;
  return GSVK_OK;
}

}  // extern "C"

namespace gsvk {

// conv_pre and the upsampling stages (dec.hpp:267-300): reads in16, leaves
// lrelu(conv_post input) in a16.  Every conv after the first is a
// programmatic dependent of its predecessor; the last conv of each residual
// block folds the block average into its epilogue (sum = cur * 1/3, then
// sum += cur * 1/3 for the later blocks: mul_write / add_scaled_inplace,
// dec.hpp:295-333).
static int decoder_body(gsvk_decoder* h, size_t T, cudaStream_t st, int* launches) {
  const gsvk_decoder_config& c = h->cfg;
  auto conv = [&](int idx, const uint16_t* x, size_t Tin, int dil, bool convt,
                  gsvk_conv_args& a, ConvFuse f) -> int {
    a.x = x;
    a.T = Tin;
    a.ci = (size_t)h->ci[idx];
    a.w = h->w[idx];
    a.co = (size_t)h->co[idx];
    a.k = (size_t)h->kk[idx];
    a.dil = (size_t)dil;
    a.bias = h->b[idx];
    f.pdl = idx > 0;
    ++*launches;
    return convt ? convt1d_run(&a, st, &f) : conv1d_run(&a, st, &f);
  };
  int rc;
  // conv_pre -> lrelu(0.1) as the first ConvT input (dec.hpp:267, 285)
  {
    gsvk_conv_args a{};
    a.y_f16_act = h->a16;
    a.act2 = GSVK_ACT_LEAKY;
    a.slope2 = c.lrelu_slope;
    if ((rc = conv(0, h->in16, T, 1, false, a, ConvFuse{}))) return rc;
  }
  size_t L = T;
  for (int s = 0; s < c.n_stages; ++s) {
    const int base = 1 + s * 19;
    const size_t Ln = L * (size_t)c.up_rate[s];
    const float next_slope = (s + 1 < c.n_stages) ? c.lrelu_slope : c.post_slope;
    {  // ConvT: xu (fp32 resblock base) and lrelu(xu) fp16
      gsvk_conv_args a{};
      a.y = h->xu32;
      a.y_f16_act = h->xu16;
      a.act2 = GSVK_ACT_LEAKY;
      a.slope2 = c.lrelu_slope;
      if ((rc = conv(base, h->a16, L, c.up_rate[s], true, a, ConvFuse{}))) return rc;
    }
    for (int j = 0; j < 3; ++j) {
      for (int p = 0; p < 3; ++p) {
        const int i1 = base + 1 + j * 6 + p * 2;
        {  // t_a = lrelu(c1(lrelu(cur)) + b) in fp16
          gsvk_conv_args a{};
          a.y_f16 = h->t16a;
          a.act = GSVK_ACT_LEAKY;
          a.slope = c.lrelu_slope;
          if ((rc = conv(i1, p == 0 ? h->xu16 : h->t16b, Ln, c.res_dil[p], false, a, ConvFuse{})))
            return rc;
        }
        {  // cur = cur + c2(t_a) + b ; next c1 input lrelu(cur) in fp16
          gsvk_conv_args a{};
          a.residual = p == 0 ? h->xu32 : h->cur32;
          a.res_scale = 1.f;
          ConvFuse f;
          if (p < 2) {
            a.y = h->cur32;
            a.y_f16_act = h->t16b;
            a.act2 = GSVK_ACT_LEAKY;
            a.slope2 = c.lrelu_slope;
          } else {
            // block output: sum += cur / 3; after the last block the next
            // stage's input lrelu(sum) in fp16
            f.mean_sum = h->sum32;
            f.mean_scale = 1.f / 3.f;
            f.mean_first = j == 0;
            if (j == 2) {
              a.y_f16_act = h->a16;
              a.act2 = GSVK_ACT_LEAKY;
              a.slope2 = next_slope;
            }
          }
          if ((rc = conv(i1 + 1, h->t16a, Ln, 1, false, a, f))) return rc;
        }
      }
    }
    L = Ln;
  }
  return GSVK_OK;
}

static int decoder_graph(gsvk_decoder* h, size_t T, cudaGraphExec_t* exec, int* launches) {
  for (auto& g : h->graphs)
    if (g.T == T) {
      g.used = ++h->tick;
      *exec = g.exec;
      *launches = g.launches;
      return GSVK_OK;
    }
  int n = 0;
  if (int rc = check_cuda(cudaStreamBeginCapture(h->capture, cudaStreamCaptureModeRelaxed),
                          "decoder capture"))
    return rc;
  const int rc_body = decoder_body(h, T, h->capture, &n);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(h->capture, &graph);
  if (rc_body || ce != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc_body ? rc_body : check_cuda(ce, "decoder capture end");
  }
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&ex, graph, 0);
  cudaGraphDestroy(graph);
  if (int rc = check_cuda(ie, "decoder graph instantiate")) return rc;
  if (h->graphs.size() >= gsvk_decoder::kMaxGraphs) {  // evict the least recently used
    auto lru = std::min_element(h->graphs.begin(), h->graphs.end(),
                                [](const auto& a, const auto& b) { return a.used < b.used; });
    cudaGraphExecDestroy(lru->exec);
    h->graphs.erase(lru);
  }
  h->graphs.push_back({T, ex, n, ++h->tick});
  *exec = ex;
  *launches = n;
  return GSVK_OK;
}

}  // namespace gsvk

extern "C" {

int gsvk_decoder_forward(gsvk_decoder_t h, const float* z, size_t T, float* wav,
                         gsvk_stream_t stream) {
  if (!h || !z || !wav || T == 0) return fail(GSVK_ERR_INVALID, "decoder_forward: null or empty");
  if (T > h->max_frames)
    return fail(GSVK_ERR_INVALID, "decoder_forward: %zu frames > max_frames %zu", T, h->max_frames);
  const gsvk_decoder_config& c = h->cfg;
  cudaStream_t st = as_cuda(stream);
  int rc = gsvk_channels_to_rows_f16(z, c.in_ch, T, h->in16, stream);
  if (rc) return rc;
  int launches = 1, body = 0;
  if (h->use_graph) {
    cudaGraphExec_t exec = nullptr;
    if ((rc = decoder_graph(h, T, &exec, &body))) return rc;
    if ((rc = check_cuda(cudaGraphLaunch(exec, st), "decoder graph launch"))) return rc;
  } else if ((rc = decoder_body(h, T, st, &body))) {
    return rc;
  }
  launches += body;
  {  // conv_post (no bias) -> tanh, written as [T_out, 1] == wav
    gsvk_conv_args a{};
    a.x = h->a16;
    a.T = gsvk_decoder_out_len(&c, T);
    const int idx = 1 + 19 * c.n_stages;
    a.ci = (size_t)h->ci[idx];
    a.w = h->w[idx];
    a.co = (size_t)h->co[idx];
    a.k = (size_t)h->kk[idx];
    a.dil = 1;
    a.bias = h->b[idx];
    a.y = wav;
    a.act = GSVK_ACT_TANH;
    if ((rc = conv1d_run(&a, st))) return rc;
    ++launches;
  }
  h->launches = launches;
  return GSVK_OK;
}

int gsvk_decoder_set_graph(gsvk_decoder_t h, int enable) {
  if (!h) return fail(GSVK_ERR_INVALID, "decoder_set_graph: null handle");
  h->use_graph = enable != 0;
  return GSVK_OK;
}

int gsvk_decoder_launches(gsvk_decoder_t h) { return h ? h->launches : 0; }

}  // extern "C"
