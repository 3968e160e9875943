// encoder.cu — post-LN transformer encoder stack: RoBERTa-large (BertLayer,
// bert_ops.hpp:347-400) and HuBERT-base (hubert.cpp:590-730) share it.
//
// Per layer, all products on the tensor-core kernel (gemm_tc.cuh):
//   qkv16 = f16(x) . Wqkv^T + b                   (q, k, v Linear fused, fp16 out)
//   S     = (Q_h K_h^T) * 1/sqrt(dh)              (batched over utterance x head)
//   P     = softmax(S + key mask) -> fp16         (bert_ops.hpp:28-43, :373-374)
//   ctx16 = P . V_h                               (batched; V_h^T packed per head)
//   y     = ctx16 . Wo^T + b + x ; x1 = LN(y)     (residual fused in the epilogue)
//   mid16 = GELU(x1 . Wi^T + b)                   (GELU fused)
//   f     = mid16 . Wf^T + b + x1 ; x = LN(f)
// The reference runs q/k/v and the attention products in fp32 (sgemm); here
// they are fp16 operands with fp32 accumulation, checked against the oracle
// at the encoder tolerance.
#include <cmath>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_encoder;

namespace gsvk {

namespace {

// Row softmax of S (fp32, ld) with keys >= valid masked by finfo.min, written
// as fp16 P (ld) with the padding columns [T, ldp) zeroed.  One warp per row.
__global__ void enc_softmax_kernel(const float* __restrict__ S, int ld, int rows, int T, int H,
                                   const int* __restrict__ valid, uint16_t* __restrict__ P) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int b = row / (H * T);
  const int nv = valid ? valid[b] : T;
  const float* s = S + static_cast<size_t>(row) * ld;
  float v[8];
  float mx = -INFINITY;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int j = lane + 32 * u;
    float x = -INFINITY;
    if (j < T) {
      x = s[j];
      if (j >= nv) x = x + -3.40282347e+38f;
    }
    v[u] = x;
    mx = fmaxf(mx, x);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int j = lane + 32 * u;
    const float e = j < T ? expf(v[u] - mx) : 0.f;
    v[u] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  uint16_t* p = P + static_cast<size_t>(row) * ld;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int j = lane + 32 * u;
    if (j < ld) p[j] = j < T ? f2h(v[u] * inv) : 0;
  }
}

// V_h^T per (utterance, head): vt[(b*H + h)*dh + d][j] = V[b*T + j][h*dh + d],
// zero for j in [T, ldt).
__global__ void enc_vt_kernel(const uint16_t* __restrict__ qkv, int C, int T, int H, int dh,
                              int ldt, uint16_t* __restrict__ vt) {
  __shared__ uint16_t tile[32][33];
  const int bh = blockIdx.z, b = bh / H, h = bh - (bh / H) * H;
  const int j0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int j = j0 + i, d = d0 + threadIdx.x;
    tile[i][threadIdx.x] = (j < T && d < dh)
                               ? qkv[(static_cast<size_t>(b) * T + j) * 3 * C + 2 * C + h * dh + d]
                               : 0;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int d = d0 + i, j = j0 + threadIdx.x;
    if (d < dh && j < ldt)
      vt[(static_cast<size_t>(bh) * dh + d) * ldt + j] = tile[threadIdx.x][i];
  }
}

// Row LayerNorm (biased variance, fp64 combine) writing fp32 and fp16.
__global__ void enc_ln_kernel(const float* __restrict__ x, const float* __restrict__ g,
                              const float* __restrict__ bta, float* __restrict__ y,
                              uint16_t* __restrict__ y16, int n, double eps) {
  __shared__ double sh[32];
  const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
  float s = 0.f, q = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i];
    s += v;
    q = fmaf(v, v, q);
  }
  double ds = warp_sum_d(static_cast<double>(s)), dq = warp_sum_d(static_cast<double>(q));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sh[w] = ds;
    sh[16 + w] = dq;
  }
  __syncthreads();
  ds = lane < nw ? sh[lane] : 0.0;
  dq = lane < nw ? sh[16 + lane] : 0.0;
  ds = warp_sum_d(ds);
  dq = warp_sum_d(dq);
  const double dn = n;
  const float mean = static_cast<float>(ds / dn);
  float var = static_cast<float>(dq / dn - static_cast<double>(mean) * mean);
  if (!(var >= 0.f)) var = 0.f;
  const float rstd = static_cast<float>(1.0 / sqrt(static_cast<double>(var) + eps));
  float* yr = y + static_cast<size_t>(blockIdx.x) * n;
  uint16_t* y16r = y16 + static_cast<size_t>(blockIdx.x) * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = fmaf((xr[i] - mean) * rstd, g[i], bta[i]);
    yr[i] = v;
    y16r[i] = f2h(v);
  }
}

// Fused attention for one (utterance b, head h, 128-query block qb), head
// dim 64, T <= 256 keys (Tp = T rounded up to 64):
//   S = Q K^T on the tensor cores into TMEM (M = 128 queries, N = Tp keys);
//   each thread owns one query row (its TMEM lane) and makes three passes
//   over it — max, sum of exp, write — producing the same fp16
//   P = softmax(S / sqrt(64)) as enc_softmax_kernel (keys >= valid[b] get
//   finfo.min added; keys >= T are dropped) straight into shared memory in
//   the 128-byte-swizzled K-major layout the MMA reads;
//   O = P V (A = P, B = V^T from enc_vt_kernel) into TMEM; fp16 O rows go to
//   the head's 64 columns of ctx.
// One thread issues the TMA loads and the MMAs and alone polls their
// mbarriers; the others wait at CTA barriers.
constexpr int kAttnDh = 64;
constexpr int kAttnQ = 128;

__device__ __forceinline__ uint32_t sw128_offset(int row, int col) {
  // byte offset of element (row, col) in a [rows][64] fp16 tile with the
  // 128-byte swizzle: 16-byte chunk index XOR (row mod 8)
  return static_cast<uint32_t>(row) * 128u +
         ((static_cast<uint32_t>(col >> 3) ^ static_cast<uint32_t>(row & 7)) << 4) +
         static_cast<uint32_t>(col & 7) * 2u;
}

constexpr int kAttnThreads = 512;  // 16 warps: four per TMEM lane quadrant

__global__ void __launch_bounds__(kAttnThreads, 1)
    enc_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmVt, int T, int Tp, int H, int C,
                    const int* __restrict__ valid, uint16_t* __restrict__ ctx, uint32_t* status) {
  extern __shared__ uint8_t at_raw[];
  uint8_t* smem = align_smem<1024>(at_raw);
  __shared__ uint64_t load_bar, s_bar, o_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ float red[8 * kAttnQ];  // per-group row max [4][128], row sum [4][128]
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkc = Tp / 64;                       // 64-key regions
  uint8_t* sVt = smem;                           // nkc x [64][64]   8 KB each
  uint8_t* sQ = sVt + nkc * 64 * 128;            // [128][64]        16 KB
  uint8_t* sK = sQ + kAttnQ * 128;               // [Tp][64]         Tp*128 B
  uint8_t* sP = sQ;                              // nkc x [128][64]  16 KB each, over Q and K
                                                 // (written once the S MMA has read them)
  // S takes columns [0, Tp); O reuses [0, 64) after the softmax has read S
  const uint32_t tmem_cols = Tp <= 64 ? 64u : (Tp <= 128 ? 128u : 256u);
  const uint32_t o_col = 0;

  if (tid == 0) {
    mbar_init(&load_bar, 1);
    mbar_init(&s_bar, 1);
    mbar_init(&o_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  griddep_wait();  // q|k|v and V^T come from the previous kernel (no-op for an ordinary launch)
  griddep_launch_dependents();
  const int row0 = b * T;  // first token row of utterance b
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmVt);
      mbar_arrive_expect_tx(&load_bar,
                            static_cast<uint32_t>(kAttnQ * 128 + Tp * 128 + nkc * 64 * 128));
      tma_load_2d(sQ, &tmQ, &load_bar, h * kAttnDh, row0 + qb * kAttnQ);
      tma_load_2d(sK, &tmK, &load_bar, C + h * kAttnDh, row0);
      for (int kc = 0; kc < nkc; ++kc)
        tma_load_2d(sVt + kc * 64 * 128, &tmVt, &load_bar, kc * 64, (b * H + h) * kAttnDh);
      bool ok = mbar_wait(&load_bar, 0, status);
      if (ok) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(sQ), b0 = smem_u32(sK);
        const uint32_t idesc = idesc_f16_f32(kAttnQ, static_cast<uint32_t>(Tp));
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc_mma_f16(tmem, smem_desc(a0 + 32u * j, 1024, 2), smem_desc(b0 + 32u * j, 1024, 2), idesc,
                     j ? 1u : 0u);
        tc_commit(&s_bar);
        mbar_wait(&s_bar, 0, status);
      }
    }
    __syncwarp();
  }
  __syncthreads();
  tc_fence_after();
  // ---------------------------------------------------------------- softmax
  // Four warps per TMEM lane quadrant: warp w serves rows 32*(w%4) .. +31 and
  // key columns [g*cw, (g+1)*cw) with g = w / 4; row max and sum are combined
  // across the four groups through shared memory (in group order).
  const int quad = warp & 3, grp = warp >> 2;
  const int r = quad * 32 + lane;  // query row within the block (TMEM lane)
  const int q = qb * kAttnQ + r;
  const int cw = Tp / 4, cbeg = grp * cw;
  const int nv = valid ? valid[b] : T;
  const uint32_t t_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
  constexpr float kScale = 0.125f;  // 1 / sqrt(64)
  // pass 1: row max.  Chunks wholly inside the valid keys skip the masks.
  const int kfull = nv < T ? nv : T;  // keys [0, kfull) need no mask
  float mx = -INFINITY;
  for (int c0 = cbeg; c0 < cbeg + cw; c0 += 16) {
    uint32_t v[16];
    tmem_ld16(t_row + static_cast<uint32_t>(c0), v);
    tmem_ld_wait();
    if (c0 + 16 <= kfull) {
#pragma unroll
      for (int j = 0; j < 16; ++j) mx = fmaxf(mx, __uint_as_float(v[j]) * kScale);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int k = c0 + j;
        float x = __uint_as_float(v[j]) * kScale;
        if (k >= nv) x = x + -3.40282347e+38f;
        if (k < T) mx = fmaxf(mx, x);
      }
    }
  }
  red[grp * kAttnQ + r] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[r], red[kAttnQ + r]), fmaxf(red[2 * kAttnQ + r], red[3 * kAttnQ + r]));
  // pass 2: e = exp(x - max) written as fp16 P (unnormalised; O is scaled by
  // 1 / sum in the epilogue) while the row sum accumulates
  float sum = 0.f;
  for (int c0 = cbeg; c0 < cbeg + cw; c0 += 16) {
    uint32_t v[16];
    tmem_ld16(t_row + static_cast<uint32_t>(c0), v);
    tmem_ld_wait();
    float e[16];
    if (c0 + 16 <= kfull) {
#pragma unroll
      for (int j = 0; j < 16; ++j) e[j] = __expf(fmaf(__uint_as_float(v[j]), kScale, -mx));
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int k = c0 + j;
        float x = __uint_as_float(v[j]) * kScale;
        if (k >= nv) x = x + -3.40282347e+38f;
        e[j] = k < T ? __expf(x - mx) : 0.f;
      }
    }
    uint32_t pk[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sum += e[2 * j] + e[2 * j + 1];
      pk[j] = f2h2(e[2 * j], e[2 * j + 1]);
    }
    uint8_t* region = sP + (c0 >> 6) * (kAttnQ * 128);
    const int cc = c0 & 63;  // 16 keys = two 16-byte chunks
    *reinterpret_cast<uint4*>(region + sw128_offset(r, cc)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    *reinterpret_cast<uint4*>(region + sw128_offset(r, cc + 8)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
  red[4 * kAttnQ + grp * kAttnQ + r] = sum;
  fence_proxy_async_shared();  // P (generic writes) -> visible to the tensor core
  tc_fence_before();
  __syncthreads();
  // ------------------------------------------------------------------ P . V
  if (tid == 0) {
    tc_fence_after();
    const uint32_t idesc = idesc_f16_f32(kAttnQ, kAttnDh);
    for (int kc = 0; kc < nkc; ++kc) {
      const uint32_t a0 = smem_u32(sP + kc * kAttnQ * 128), b0 = smem_u32(sVt + kc * 64 * 128);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc_mma_f16(tmem + o_col, smem_desc(a0 + 32u * j, 1024, 2), smem_desc(b0 + 32u * j, 1024, 2),
                   idesc, (kc | j) ? 1u : 0u);
    }
    tc_commit(&o_bar);
    mbar_wait(&o_bar, 0, status);
  }
  __syncthreads();
  tc_fence_after();
  {  // group g stores O columns [16 g, 16 g + 16) of its rows, scaled by 1 / row sum
    const float* rs = red + 4 * kAttnQ;
    const float inv = 1.f / (((rs[r] + rs[kAttnQ + r]) + rs[2 * kAttnQ + r]) + rs[3 * kAttnQ + r]);
    uint32_t v[16];
    tmem_ld16(t_row + o_col + 16u * static_cast<uint32_t>(grp), v);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * inv);
    if (q < T) {
      uint4* dst = reinterpret_cast<uint4*>(ctx + static_cast<size_t>(row0 + q) * C + h * kAttnDh +
                                            16 * grp);
      uint32_t pk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pk[j] = f2h2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

size_t enc_attn_smem(int Tp) {
  const size_t qk = static_cast<size_t>(kAttnQ) * 128 + static_cast<size_t>(Tp) * 128;
  const size_t p = static_cast<size_t>(Tp / 64) * kAttnQ * 128;
  return 1024 + static_cast<size_t>(Tp / 64) * 64 * 128 + (qk > p ? qk : p);
}

// Row LayerNorm, one warp per row of n = 128 * NV4 values: every lane reads
// its NV4 float4 slices once (coalesced), sums them in fp32, and the warp
// combines the partial sums in fp64 (the reference's fp64 statistics);
// normalised values go out as fp32 and fp16 from the same registers.
template <int NV4>
__global__ void __launch_bounds__(256) enc_ln_warp_kernel(const float* __restrict__ x,
                                                          const float* __restrict__ g,
                                                          const float* __restrict__ bta,
                                                          float* __restrict__ y,
                                                          uint16_t* __restrict__ y16, int rows,
                                                          double eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  griddep_wait();  // x comes from the previous kernel (no-op for an ordinary launch)
  griddep_launch_dependents();
  if (row >= rows) return;
  constexpr int n = NV4 * 128;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * n);
  float4 v[NV4];
  float s = 0.f, q = 0.f;
#pragma unroll
  for (int u = 0; u < NV4; ++u) v[u] = xr[lane + 32 * u];
#pragma unroll
  for (int u = 0; u < NV4; ++u) {
    s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
    q = fmaf(v[u].x, v[u].x, q);
    q = fmaf(v[u].y, v[u].y, q);
    q = fmaf(v[u].z, v[u].z, q);
    q = fmaf(v[u].w, v[u].w, q);
  }
  const double ds = warp_sum_d(static_cast<double>(s)), dq = warp_sum_d(static_cast<double>(q));
  const float mean = static_cast<float>(ds / n);
  float var = static_cast<float>(dq / n - static_cast<double>(mean) * mean);
  if (!(var >= 0.f)) var = 0.f;
  const float rstd = static_cast<float>(1.0 / sqrt(static_cast<double>(var) + eps));
  float4* yr = reinterpret_cast<float4*>(y + static_cast<size_t>(row) * n);
  uint2* y16r = reinterpret_cast<uint2*>(y16 + static_cast<size_t>(row) * n);
#pragma unroll
  for (int u = 0; u < NV4; ++u) {
    const int i = lane + 32 * u;
    const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + i);
    const float4 bb = __ldg(reinterpret_cast<const float4*>(bta) + i);
    float4 o;
    o.x = fmaf((v[u].x - mean) * rstd, gg.x, bb.x);
    o.y = fmaf((v[u].y - mean) * rstd, gg.y, bb.y);
    o.z = fmaf((v[u].z - mean) * rstd, gg.z, bb.z);
    o.w = fmaf((v[u].w - mean) * rstd, gg.w, bb.w);
    yr[i] = o;
    y16r[i] = make_uint2(f2h2(o.x, o.y), f2h2(o.z, o.w));
  }
}

// pdl: launched as a programmatic dependent of the previous kernel (the warp
// kernel waits for it before reading x).
int enc_layernorm(const float* x, const float* g, const float* b, float* y, uint16_t* y16, int rows,
                  int n, double eps, cudaStream_t st, bool pdl) {
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  switch (n % 128 == 0 ? n / 128 : 0) {
#define GSVK_LN_CASE(K)                                                                   \
  case K:                                                                                 \
    if (pdl)                                                                              \
      return launch_pdl(enc_ln_warp_kernel<K>, dim3(blocks), dim3(256), 0, st,            \
                        "enc_ln_warp_kernel", x, g, b, y, y16, rows, eps);                \
    enc_ln_warp_kernel<K><<<blocks, 256, 0, st>>>(x, g, b, y, y16, rows, eps);            \
    return check_launch("enc_ln_warp_kernel");
    GSVK_LN_CASE(4) GSVK_LN_CASE(5) GSVK_LN_CASE(6) GSVK_LN_CASE(7) GSVK_LN_CASE(8)
    GSVK_LN_CASE(10) GSVK_LN_CASE(12) GSVK_LN_CASE(16)
#undef GSVK_LN_CASE
    default:
      enc_ln_kernel<<<static_cast<unsigned>(rows), 256, 0, st>>>(x, g, b, y, y16, n, eps);
      return check_launch("enc_ln_kernel");
  }
}

}  // namespace

struct EncoderEngine {
  gsvk_encoder_config cfg{};
  void* wmem = nullptr;
  void* amem = nullptr;
  const uint16_t *wqkv = nullptr, *wo = nullptr, *wi = nullptr, *wf = nullptr;
  const float *bqkv = nullptr, *bo = nullptr, *bi = nullptr, *bf = nullptr;
  const float *ln1g = nullptr, *ln1b = nullptr, *ln2g = nullptr, *ln2b = nullptr;
  uint16_t *x16 = nullptr, *qkv16 = nullptr, *p16 = nullptr, *vt16 = nullptr, *ctx16 = nullptr,
           *x1_16 = nullptr, *mid16 = nullptr;
  float *s32 = nullptr, *y32 = nullptr, *x1_32 = nullptr, *f32 = nullptr;
  int launches = 0;
};

}  // namespace gsvk

using namespace gsvk;

struct gsvk_encoder : gsvk::EncoderEngine {};

extern "C" {

int gsvk_encoder_destroy(gsvk_encoder_t h) {
  if (!h) return GSVK_OK;
  if (h->wmem) cudaFree(h->wmem);
  if (h->amem) cudaFree(h->amem);
  delete h;
  return GSVK_OK;
}

int gsvk_encoder_create(const gsvk_encoder_config* cfg, const gsvk_encoder_host_weights* w,
                        gsvk_encoder_t* out) {
  if (!cfg || !w || !out) return fail(GSVK_ERR_INVALID, "encoder_create: null argument");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  const int L = cfg->layers, C = cfg->hidden, H = cfg->heads, F = cfg->ffn;
  if (L <= 0 || C <= 0 || H <= 0 || F <= 0 || C % H || cfg->max_batch <= 0 || cfg->max_seq <= 0)
    return fail(GSVK_ERR_INVALID, "encoder_create: bad dimensions");
  const int dh = C / H;
  if (dh % 64 || C % 64 || F % 64 || cfg->max_seq > 256)
    return fail(GSVK_ERR_UNSUPPORTED,
                "encoder_create: head_dim, hidden and ffn must be multiples of 64, seq <= 256");
  auto* e = new gsvk_encoder();
  e->cfg = *cfg;
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t nqkv = (size_t)L * 3 * C * C, no = (size_t)L * C * C, ni = (size_t)L * F * C,
               nf = (size_t)L * C * F;
  struct Up { size_t off; const void* src; size_t bytes; };
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al(bytes); return o; };
  const size_t o_wqkv = take(nqkv * 2), o_wo = take(no * 2), o_wi = take(ni * 2),
               o_wf = take(nf * 2), o_bqkv = take((size_t)L * 3 * C * 4),
               o_bo = take((size_t)L * C * 4), o_bi = take((size_t)L * F * 4),
               o_bf = take((size_t)L * C * 4), o_l1g = take((size_t)L * C * 4),
               o_l1b = take((size_t)L * C * 4), o_l2g = take((size_t)L * C * 4),
               o_l2b = take((size_t)L * C * 4);
  if (cudaMalloc(&e->wmem, off) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return fail(GSVK_ERR_NOMEM, "encoder_create: weights");
  }
  uint8_t* base = static_cast<uint8_t*>(e->wmem);
  const Up ups[] = {{o_wqkv, w->wqkv, nqkv * 2}, {o_wo, w->wo, no * 2}, {o_wi, w->wi, ni * 2},
                    {o_wf, w->wf, nf * 2}, {o_bqkv, w->bqkv, (size_t)L * 3 * C * 4},
                    {o_bo, w->bo, (size_t)L * C * 4}, {o_bi, w->bi, (size_t)L * F * 4},
                    {o_bf, w->bf, (size_t)L * C * 4}, {o_l1g, w->ln1g, (size_t)L * C * 4},
                    {o_l1b, w->ln1b, (size_t)L * C * 4}, {o_l2g, w->ln2g, (size_t)L * C * 4},
                    {o_l2b, w->ln2b, (size_t)L * C * 4}};
  for (const Up& u : ups) {
    if (!u.src) {
      gsvk_encoder_destroy(e);
      return fail(GSVK_ERR_INVALID, "encoder_create: null weight");
    }
    int rc = check_cuda(cudaMemcpy(base + u.off, u.src, u.bytes, cudaMemcpyHostToDevice),
                        "encoder upload");
    if (rc) { gsvk_encoder_destroy(e); return rc; }
  }
  e->wqkv = reinterpret_cast<const uint16_t*>(base + o_wqkv);
  e->wo = reinterpret_cast<const uint16_t*>(base + o_wo);
  e->wi = reinterpret_cast<const uint16_t*>(base + o_wi);
  e->wf = reinterpret_cast<const uint16_t*>(base + o_wf);
  e->bqkv = reinterpret_cast<const float*>(base + o_bqkv);
  e->bo = reinterpret_cast<const float*>(base + o_bo);
  e->bi = reinterpret_cast<const float*>(base + o_bi);
  e->bf = reinterpret_cast<const float*>(base + o_bf);
  e->ln1g = reinterpret_cast<const float*>(base + o_l1g);
  e->ln1b = reinterpret_cast<const float*>(base + o_l1b);
  e->ln2g = reinterpret_cast<const float*>(base + o_l2g);
  e->ln2b = reinterpret_cast<const float*>(base + o_l2b);
  // activations for max_batch x max_seq tokens
  const size_t M = (size_t)cfg->max_batch * cfg->max_seq;
  const size_t Tp = ((size_t)cfg->max_seq + 63) / 64 * 64;
  const size_t BHT = (size_t)cfg->max_batch * H * cfg->max_seq;
  off = 0;
  const size_t o_x16 = take(M * C * 2), o_qkv = take(M * 3 * C * 2), o_s = take(BHT * Tp * 4),
               o_p = take(BHT * Tp * 2), o_vt = take((size_t)cfg->max_batch * H * dh * Tp * 2),
               o_ctx = take(M * C * 2), o_y = take(M * C * 4), o_x1 = take(M * C * 4),
               o_x116 = take(M * C * 2), o_mid = take(M * F * 2), o_f = take(M * C * 4);
  if (cudaMalloc(&e->amem, off) != cudaSuccess) {
    cudaGetLastError();
    gsvk_encoder_destroy(e);
    return fail(GSVK_ERR_NOMEM, "encoder_create: activations (%zu bytes)", off);
  }
  // zeroed once: the padding keys of V^T (columns T .. Tp of each row) are
  // never written by the q|k|v epilogue, and P is exactly 0 there
  if (int rc = check_cuda(cudaMemset(e->amem, 0, off), "encoder activations memset")) {
    gsvk_encoder_destroy(e);
    return rc;
  }
  uint8_t* a = static_cast<uint8_t*>(e->amem);
  e->x16 = reinterpret_cast<uint16_t*>(a + o_x16);
  e->qkv16 = reinterpret_cast<uint16_t*>(a + o_qkv);
  e->s32 = reinterpret_cast<float*>(a + o_s);
  e->p16 = reinterpret_cast<uint16_t*>(a + o_p);
  e->vt16 = reinterpret_cast<uint16_t*>(a + o_vt);
  e->ctx16 = reinterpret_cast<uint16_t*>(a + o_ctx);
  e->y32 = reinterpret_cast<float*>(a + o_y);
  e->x1_32 = reinterpret_cast<float*>(a + o_x1);
  e->x1_16 = reinterpret_cast<uint16_t*>(a + o_x116);
  e->mid16 = reinterpret_cast<uint16_t*>(a + o_mid);
  e->f32 = reinterpret_cast<float*>(a + o_f);
  *out = e;
  return GSVK_OK;
}

int gsvk_encoder_forward(gsvk_encoder_t h, float* x, size_t batch, size_t seq, const int* valid,
                         gsvk_stream_t stream) {
  if (!h || !x || batch == 0 || seq == 0) return fail(GSVK_ERR_INVALID, "encoder_forward: null");
  if (batch > (size_t)h->cfg.max_batch || seq > (size_t)h->cfg.max_seq)
    return fail(GSVK_ERR_INVALID, "encoder_forward: batch/seq exceed the handle's maxima");
  const gsvk_encoder_config& c = h->cfg;
  const int C = c.hidden, H = c.heads, F = c.ffn, dh = C / H, T = (int)seq, B = (int)batch;
  const int M = B * T, Tp = (T + 63) / 64 * 64;
  // fused tensor-core attention covers head dim 64 and up to 256 keys
  const bool fused = dh == kAttnDh && Tp <= 256;
  if (fused) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
      if (int rc0 = check_cuda(cudaFuncSetAttribute(enc_attn_kernel,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    (int)enc_attn_smem(256)),
                               "cudaFuncSetAttribute(enc_attn)"))
        return rc0;
      attr_set[dev] = true;
    }
  }
  cudaStream_t st = as_cuda(stream);
  int launches = 0;
  int rc = gsvk_f32_to_f16(x, h->x16, (size_t)M * C, stream);
  if (rc) return rc;
  ++launches;
  auto gemm = [&](const uint16_t* A, int lda, const uint16_t* W, int N, int K, const float* bias,
                  int act, const float* res, float* c32, uint16_t* c16) -> int {
    gsvk_gemm_args g{};
    g.a = A;
    g.lda = lda;
    g.b = W;
    g.ldb = K;
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.act = act;
    g.residual = res;
    g.ld_res = N;
    g.c = c32;
    g.ldc = N;
    g.c_f16 = c16;
    g.ldc_f16 = N;
    g.alpha = 1.f;
    ++launches;
    return gemm_ex_run(&g, st, fused);
  };
  for (int l = 0; l < c.layers; ++l) {
    // q|k|v (with the fused attention, V goes out transposed per head: V^T is
    // the B operand of P.V)
    if (fused) {
      TcProblem p{};
      p.M = M;
      p.N = 3 * C;
      p.kc = C;
      p.taps = 1;
      p.dil = 1;
      p.phases = 1;
      p.out_rows = M;
      TcEpilogue e = make_epilogue();
      e.bias = h->bqkv + (size_t)l * 3 * C;
      e.c16 = h->qkv16;
      e.ld_c16 = 3 * C;
      e.vt = h->vt16;
      e.vt_ld = Tp;
      e.vt_c0 = 2 * C;
      e.vt_T = T;
      e.vt_dh = dh;
      e.vt_H = H;
      p.pdl = 1;
      if ((rc = tc_run(h->x16, M, C, h->wqkv + (size_t)l * 3 * C * C, 3 * C, C, p, e, 0, st)))
        return rc;
      ++launches;
    } else if ((rc = gemm(h->x16, C, h->wqkv + (size_t)l * 3 * C * C, 3 * C, C,
                          h->bqkv + (size_t)l * 3 * C, GSVK_ACT_NONE, nullptr, nullptr, h->qkv16))) {
      return rc;
    }
    if (fused) {
      // S, softmax and P V in one kernel (V^T came from the q|k|v epilogue)
      CUtensorMap tq, tk, tv;
      if ((rc = make_kmajor_map(&tq, h->qkv16, M, 3 * C, 3 * C, kAttnQ, 64))) return rc;
      if ((rc = make_kmajor_map(&tk, h->qkv16, M, 3 * C, 3 * C, Tp, 64))) return rc;
      if ((rc = make_kmajor_map(&tv, h->vt16, (long long)B * H * dh, Tp, Tp, 64, 64))) return rc;
      if ((rc = launch_pdl(enc_attn_kernel,
                           dim3((unsigned)((T + kAttnQ - 1) / kAttnQ), (unsigned)H, (unsigned)B),
                           dim3(kAttnThreads), enc_attn_smem(Tp), st, "enc_attn_kernel", tq, tk,
                           tv, T, Tp, H, C, valid, h->ctx16, device_status())))
        return rc;
      ++launches;
    } else {
      // S = Q K^T / sqrt(dh), batched over (utterance, head)
      {
        TcProblem p{};
        p.M = T;
        p.N = T;
        p.kc = dh;
        p.taps = 1;
        p.dil = 1;
        p.phases = B * H;
        p.out_rows = T;
        p.bh = H;
        p.a_rb = T; p.a_rh = 0; p.a_ch = dh; p.a_c0 = 0;
        p.b_rb = T; p.b_rh = 0; p.b_ch = dh; p.b_c0 = C;
        p.c_rb = H * T; p.c_rh = T; p.c_ch = 0;
        TcEpilogue e = make_epilogue();
        e.alpha = 1.f / std::sqrt(static_cast<float>(dh));
        e.c32 = h->s32;
        e.ld_c32 = Tp;
        if ((rc = tc_run(h->qkv16, M, 3 * C, h->qkv16, M, 3 * C, p, e, 0, st, 3 * C, 3 * C)))
          return rc;
        ++launches;
      }
      {
        const int rows = B * H * T;
        enc_softmax_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(h->s32, Tp, rows, T,
                                                                              H, valid, h->p16);
        if ((rc = check_launch("enc_softmax_kernel"))) return rc;
        dim3 grid((unsigned)((Tp + 31) / 32), (unsigned)((dh + 31) / 32), (unsigned)(B * H));
        enc_vt_kernel<<<grid, dim3(32, 8), 0, st>>>(h->qkv16, C, T, H, dh, Tp, h->vt16);
        if ((rc = check_launch("enc_vt_kernel"))) return rc;
        launches += 2;
      }
      // ctx = P V_h, written into the head's columns of ctx16
      {
        TcProblem p{};
        p.M = T;
        p.N = dh;
        p.kc = Tp;
        p.taps = 1;
        p.dil = 1;
        p.phases = B * H;
        p.out_rows = T;
        p.bh = H;
        p.a_rb = H * T; p.a_rh = T; p.a_ch = 0; p.a_c0 = 0;
        p.b_rb = H * dh; p.b_rh = dh; p.b_ch = 0; p.b_c0 = 0;
        p.c_rb = T; p.c_rh = 0; p.c_ch = dh;
        TcEpilogue e = make_epilogue();
        e.c16 = h->ctx16;
        e.ld_c16 = C;
        if ((rc = tc_run(h->p16, (long long)B * H * T, Tp, h->vt16, (long long)B * H * dh, Tp, p, e,
                         0, st)))
          return rc;
        ++launches;
      }
    }
    // attn_out + b + x -> LN1
    if ((rc = gemm(h->ctx16, C, h->wo + (size_t)l * C * C, C, C, h->bo + (size_t)l * C,
                   GSVK_ACT_NONE, x, h->y32, nullptr)))
      return rc;
    if ((rc = enc_layernorm(h->y32, h->ln1g + (size_t)l * C, h->ln1b + (size_t)l * C, h->x1_32,
                            h->x1_16, M, C, c.eps, st, fused)))
      return rc;
    ++launches;
    // FFN
    if ((rc = gemm(h->x1_16, C, h->wi + (size_t)l * F * C, F, C, h->bi + (size_t)l * F,
                   GSVK_ACT_GELU_ERF, nullptr, nullptr, h->mid16)))
      return rc;
    if ((rc = gemm(h->mid16, F, h->wf + (size_t)l * C * F, C, F, h->bf + (size_t)l * C,
                   GSVK_ACT_NONE, h->x1_32, h->f32, nullptr)))
      return rc;
    if ((rc = enc_layernorm(h->f32, h->ln2g + (size_t)l * C, h->ln2b + (size_t)l * C, x, h->x16, M,
                            C, c.eps, st, fused)))
      return rc;
    ++launches;
  }
  h->launches = launches;
  return GSVK_OK;
}

int gsvk_encoder_launches(gsvk_encoder_t h) { return h ? h->launches : 0; }

}  // extern "C"
