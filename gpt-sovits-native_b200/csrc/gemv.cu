// gemv.cu — decode GEMV y[out] = act(W[out,in] . x + bias) + residual.
//
// Replaces kern::gemv_f16w_f32acc (gemv.cpp:113) and kern::gemv_f16x_fmlal
// (gemv_fmlal.cpp:113).  Both are HBM-bound: W (fp16, row-major) is streamed
// once with 128-bit non-allocating loads; x (fp32 or fp16, a few KB) stays in
// L1 and is re-read by every warp.
//
// Layout of work: one warp owns R consecutive rows; each lane walks the row in
// 8-element (16-byte) chunks strided by 32 lanes, with U chunks per row issued
// back to back so that R*U 16-byte loads per lane are in flight.  The fp32
// partial sums are combined with a butterfly shuffle.  Products fp16 x fp32
// (or fp16 x fp16) are formed in fp32 exactly as the reference widens
// (vcvt_f32_f16 / FMLAL) and accumulated with fp32 FMA.
#include "common.cuh"

namespace gsvk {

namespace {

constexpr int kWarps = 8;  // 256 threads per CTA
constexpr int kU = 4;      // chunks in flight per row per lane

template <bool XF16>
__device__ __forceinline__ void load_x8(const void* x, int chunk, float* xf) {
  if constexpr (XF16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x) + chunk);
    unpack8(v, xf);
  } else {
    const float4* p = reinterpret_cast<const float4*>(x) + 2 * chunk;
    const float4 a = __ldg(p), b = __ldg(p + 1);
    xf[0] = a.x; xf[1] = a.y; xf[2] = a.z; xf[3] = a.w;
    xf[4] = b.x; xf[5] = b.y; xf[6] = b.z; xf[7] = b.w;
  }
}

template <bool XF16>
__device__ __forceinline__ float load_x1(const void* x, int i) {
  if constexpr (XF16)
    return h2f(reinterpret_cast<const uint16_t*>(x)[i]);
  else
    return reinterpret_cast<const float*>(x)[i];
}

__device__ __forceinline__ void epilogue_store(float acc, int row, float* y, uint16_t* yh,
                                               const float* bias, const float* res, int act,
                                               float slope) {
  float v = acc;
  if (bias) v = v + bias[row];
  v = apply_act(v, act, slope);
  if (res) v = v + res[row];
  if (y) y[row] = v;
  if (yh) yh[row] = f2h(v);
}

// Vector path: in % 8 == 0, W / x 16-byte aligned.
template <bool XF16, int R>
__global__ void __launch_bounds__(kWarps * 32) gemv_vec_kernel(
    const uint16_t* __restrict__ w, const void* __restrict__ x, float* __restrict__ y,
    uint16_t* __restrict__ yh, int out, int in, const float* __restrict__ bias,
    const float* __restrict__ res, int act, float slope) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * kWarps + warp) * R;
  if (row0 >= out) return;
  const int nchunk = in >> 3;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  const uint16_t* wr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) wr[r] = w + static_cast<size_t>(min(row0 + r, out - 1)) * in;

  int c = lane;
  for (; c + 32 * (kU - 1) < nchunk; c += 32 * kU) {
    uint4 wv[R][kU];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int u = 0; u < kU; ++u) wv[r][u] = ld_stream_u4(wr[r] + 8 * (c + 32 * u));
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float xf[8];
      load_x8<XF16>(x, c + 32 * u, xf);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float wf[8];
        unpack8(wv[r][u], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r] = fmaf(wf[e], xf[e], acc[r]);
      }
    }
  }
  for (; c < nchunk; c += 32) {
    float xf[8];
    load_x8<XF16>(x, c, xf);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float wf[8];
      unpack8(ld_stream_u4(wr[r] + 8 * c), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[r] = fmaf(wf[e], xf[e], acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
  if (lane < R && row0 + lane < out) {
    float a = acc[0];
#pragma unroll
    for (int r = 1; r < R; ++r)
      if (lane == r) a = acc[r];
    epilogue_store(a, row0 + lane, y, yh, bias, res, act, slope);
  }
}

// Generic path (any in, any alignment): one warp per row, scalar loads.
template <bool XF16>
__global__ void __launch_bounds__(kWarps * 32) gemv_scalar_kernel(
    const uint16_t* __restrict__ w, const void* __restrict__ x, float* __restrict__ y,
    uint16_t* __restrict__ yh, int out, int in, const float* __restrict__ bias,
    const float* __restrict__ res, int act, float slope) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + warp;
  if (row >= out) return;
  const uint16_t* wr = w + static_cast<size_t>(row) * in;
  float acc = 0.f;
  for (int i = lane; i < in; i += 32) acc = fmaf(h2f(wr[i]), load_x1<XF16>(x, i), acc);
  acc = warp_sum(acc);
  if (lane == 0) epilogue_store(acc, row, y, yh, bias, res, act, slope);
}

template <bool XF16>
int launch_gemv(const uint16_t* w, const void* x, float* y, uint16_t* yh, size_t out, size_t in,
                const float* bias, const float* res, int act, float slope, cudaStream_t st) {
  const bool vec = (in % 8 == 0) && aligned16(w) && aligned16(x);
  if (!vec) {
    gemv_scalar_kernel<XF16><<<ceil_div(out, kWarps), kWarps * 32, 0, st>>>(
        w, x, y, yh, (int)out, (int)in, bias, res, act, slope);
    return check_launch("gemv_scalar_kernel");
  }
  // Rows per warp: enough CTAs to cover every SM at least twice first, then
  // more rows per warp for more bytes in flight per lane.
  const size_t sms = static_cast<size_t>(sm_count());
  if (out >= sms * kWarps * 4 * 2) {
    gemv_vec_kernel<XF16, 4><<<ceil_div(out, kWarps * 4), kWarps * 32, 0, st>>>(
        w, x, y, yh, (int)out, (int)in, bias, res, act, slope);
  } else if (out >= sms * kWarps * 2 * 2) {
    gemv_vec_kernel<XF16, 2><<<ceil_div(out, kWarps * 2), kWarps * 32, 0, st>>>(
        w, x, y, yh, (int)out, (int)in, bias, res, act, slope);
  } else {
    gemv_vec_kernel<XF16, 1><<<ceil_div(out, kWarps), kWarps * 32, 0, st>>>(
        w, x, y, yh, (int)out, (int)in, bias, res, act, slope);
  }
  return check_launch("gemv_vec_kernel");
}

__global__ void f32_to_f16_kernel(const float* __restrict__ s, uint16_t* __restrict__ d,
                                  size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    d[i] = f2h(s[i]);
}
__global__ void f16_to_f32_kernel(const uint16_t* __restrict__ s, float* __restrict__ d,
                                  size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    d[i] = h2f(s[i]);
}

unsigned elementwise_grid(size_t n) {
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  size_t g = (n + 255) / 256;
  return static_cast<unsigned>(g < cap ? (g ? g : 1) : cap);
}

}  // namespace

int gemv_ex(const uint16_t* w, const void* x, int x_is_f16, float* y, uint16_t* yh, size_t out,
            size_t in, const float* bias, const float* residual, int act, float slope,
            cudaStream_t st) {
  if (!w || !x || (!y && !yh) || out == 0 || in == 0)
    return fail(GSVK_ERR_INVALID, "gemv: null pointer or zero size (out=%zu in=%zu)", out, in);
  if (out > 0x7fffffff || in > 0x7fffffff) return fail(GSVK_ERR_UNSUPPORTED, "gemv: size > 2^31");
  if (x_is_f16)
    return launch_gemv<true>(w, x, y, yh, out, in, bias, residual, act, slope, st);
  return launch_gemv<false>(w, x, y, yh, out, in, bias, residual, act, slope, st);
}

}  // namespace gsvk

using namespace gsvk;

extern "C" {

int gsvk_gemv_f16w_f32acc(const uint16_t* w, const float* x, float* y, size_t out, size_t in,
                          gsvk_stream_t stream) {
  if (!y) return fail(GSVK_ERR_INVALID, "gemv_f16w_f32acc: null y");
  return gemv_ex(w, x, 0, y, nullptr, out, in, nullptr, nullptr, GSVK_ACT_NONE, 0.f,
                 as_cuda(stream));
}

int gsvk_gemv_f16x_fmlal(const uint16_t* w, const uint16_t* xh, float* y, size_t out, size_t in,
                         gsvk_stream_t stream) {
  if (!y) return fail(GSVK_ERR_INVALID, "gemv_f16x_fmlal: null y");
  return gemv_ex(w, xh, 1, y, nullptr, out, in, nullptr, nullptr, GSVK_ACT_NONE, 0.f,
                 as_cuda(stream));
}

int gsvk_gemv_ex(const uint16_t* w, const void* x, int x_is_f16, float* y, uint16_t* y_f16,
                 size_t out, size_t in, const float* bias, const float* residual, int act,
                 float slope, gsvk_stream_t stream) {
  if (act < GSVK_ACT_NONE || act > GSVK_ACT_TANH) return fail(GSVK_ERR_INVALID, "gemv: bad act");
  return gemv_ex(w, x, x_is_f16, y, y_f16, out, in, bias, residual, act, slope, as_cuda(stream));
}

int gsvk_f32_to_f16(const float* src, uint16_t* dst, size_t n, gsvk_stream_t stream) {
  if (!src || !dst) return fail(GSVK_ERR_INVALID, "f32_to_f16: null pointer");
  if (n == 0) return GSVK_OK;
  f32_to_f16_kernel<<<elementwise_grid(n), 256, 0, as_cuda(stream)>>>(src, dst, n);
  return check_launch("f32_to_f16_kernel");
}

int gsvk_f16_to_f32(const uint16_t* src, float* dst, size_t n, gsvk_stream_t stream) {
  if (!src || !dst) return fail(GSVK_ERR_INVALID, "f16_to_f32: null pointer");
  if (n == 0) return GSVK_OK;
  f16_to_f32_kernel<<<elementwise_grid(n), 256, 0, as_cuda(stream)>>>(src, dst, n);
  return check_launch("f16_to_f32_kernel");
}

}  // extern "C"
