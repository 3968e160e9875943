// prims.cu — support primitives on the decode/encode critical path:
// LayerNorm (kern.cpp:27), row softmax (kern.cpp:62-77) and elementwise
// activations (kern.cpp:85, bert_ops.hpp:25, nn_ops.hpp:48).
#include "common.cuh"

namespace gsvk {

namespace {

// Block-wide sum of a double (blockDim.x a multiple of 32, <= 1024).
__device__ double block_sum_d(double v, double* sh) {
  v = warp_sum_d(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double t = lane < nw ? sh[lane] : 0.0;
  t = warp_sum_d(t);
  return t;
}
__device__ float block_max(float v, float* sh) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = lane < nw ? sh[lane] : -INFINITY;
  return warp_max(t);
}
__device__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = lane < nw ? sh[lane] : 0.f;
  return warp_sum(t);
}

// One CTA per row.  Per-thread fp32 partial sums (the reference keeps fp32
// lane sums), combined in fp64 exactly where the reference widens
// (kern.cpp:40-41); mean and biased variance then follow kern.cpp:43-53.
__global__ void layernorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                      const float* __restrict__ b, float* __restrict__ y, int n,
                                      double eps) {
  __shared__ double shd[32];
  const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
  float* yr = y + static_cast<size_t>(blockIdx.x) * n;
  float s = 0.f, q = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i];
    s += v;
    q = fmaf(v, v, q);
  }
  const double sum = block_sum_d(static_cast<double>(s), shd);
  const double sqsum = block_sum_d(static_cast<double>(q), shd);
  const double dn = static_cast<double>(n);
  const float mean = static_cast<float>(sum / dn);
  float var = static_cast<float>(sqsum / dn - static_cast<double>(mean) * mean);
  if (!(var >= 0.0f)) {
    double s2 = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const double d = static_cast<double>(xr[i]) - mean;
      s2 += d * d;
    }
    var = static_cast<float>(block_sum_d(s2, shd) / dn);
  }
  const float rstd = static_cast<float>(1.0 / sqrt(static_cast<double>(var) + eps));
  __syncthreads();  // in-place: every thread has finished reading xr
  for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = fmaf((xr[i] - mean) * rstd, g[i], b[i]);
}

__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, int n) {
  __shared__ float sh[32];
  const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
  float* yr = y + static_cast<size_t>(blockIdx.x) * n;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, xr[i]);
  m = block_max(m, sh);
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += expf(xr[i] - m);
  s = block_sum(s, sh);
  const float inv = 1.0f / s;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = expf(xr[i] - m) * inv;
}

__global__ void act_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n, int act,
                           float slope) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    y[i] = apply_act(x[i], act, slope);
}

int row_threads(size_t n) {
  if (n >= 1024) return 256;
  if (n >= 256) return 128;
  return 32;
}

}  // namespace
}  // namespace gsvk

using namespace gsvk;

extern "C" {

int gsvk_layernorm_rows(const float* x, const float* g, const float* b, float* y, size_t rows,
                        size_t n, double eps, gsvk_stream_t stream) {
  if (!x || !g || !b || !y || rows == 0 || n == 0)
    return fail(GSVK_ERR_INVALID, "layernorm_rows: null pointer or zero size");
  if (rows > 0x7fffffff || n > 0x7fffffff) return fail(GSVK_ERR_UNSUPPORTED, "layernorm: too big");
  layernorm_rows_kernel<<<(unsigned)rows, row_threads(n), 0, as_cuda(stream)>>>(x, g, b, y, (int)n,
                                                                             eps);
  return check_launch("layernorm_rows_kernel");
}

int gsvk_softmax_rows(const float* x, float* y, size_t rows, size_t n, gsvk_stream_t stream) {
  if (!x || !y || rows == 0 || n == 0)
    return fail(GSVK_ERR_INVALID, "softmax_rows: null pointer or zero size");
  if (rows > 0x7fffffff || n > 0x7fffffff) return fail(GSVK_ERR_UNSUPPORTED, "softmax: too big");
  softmax_rows_kernel<<<(unsigned)rows, row_threads(n), 0, as_cuda(stream)>>>(x, y, (int)n);
  return check_launch("softmax_rows_kernel");
}

int gsvk_activation(const float* x, float* y, size_t n, int act, float slope,
                    gsvk_stream_t stream) {
  if (!x || !y) return fail(GSVK_ERR_INVALID, "activation: null pointer");
  if (act < GSVK_ACT_NONE || act > GSVK_ACT_TANH) return fail(GSVK_ERR_INVALID, "bad act");
  if (n == 0) return GSVK_OK;
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  size_t g = (n + 255) / 256;
  if (g > cap) g = cap;
  act_kernel<<<(unsigned)g, 256, 0, as_cuda(stream)>>>(x, y, n, act, slope);
  return check_launch("act_kernel");
}

}  // extern "C"
