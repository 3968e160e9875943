// sgemm.cu — accel::sgemm (accel.hpp:22-30, accel.cpp:25-33): row-major fp32
// C = alpha * op(A) * op(B) + beta * C with op = identity ('N') or transpose
// ('T'); beta == 0 never reads C (cblas semantics, so C may hold NaN).
//
// fp32 operands on CUDA cores: the reference's contract is an fp32 GEMM
// (its tests compare against a naive fp32 loop at 1e-5), which the tf32 or
// fp16 tensor-core paths would not meet.  64 x 64 output tiles, 16-deep K
// slices staged in shared memory, 4 x 4 outputs per thread.
//
// The same kernel with fp16 B widened exactly as it is staged is
// accel::gemm_nt_f16w (accel.hpp:38-41: y = x . W^T with W [out, in] fp16):
// bit-identical to sgemm on an fp32 up-cast copy of W, without the copy.
#include "gsvk_internal.hpp"

namespace gsvk {
namespace {

constexpr int kT = 64, kK = 16;

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(uint16_t v) { return __half2float(__ushort_as_half(v)); }

template <typename TB>
__global__ void __launch_bounds__(256) sgemm_kernel(int M, int N, int K, float alpha,
                                                    const float* __restrict__ A, int lda, int ta,
                                                    const TB* __restrict__ B, int ldb, int tb,
                                                    float beta, float* __restrict__ C, int ldc) {
  __shared__ float As[kK][kT + 4];
  __shared__ float Bs[kK][kT + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kT, n0 = blockIdx.x * kT;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kK) {
    for (int i = threadIdx.x; i < kK * kT; i += 256) {
      const int kk = i / kT, mm = i % kT;
      const int m = m0 + mm, k = k0 + kk;
      float av = 0.f, bv = 0.f;
      if (m < M && k < K) av = ta ? A[static_cast<size_t>(k) * lda + m] : A[static_cast<size_t>(m) * lda + k];
      const int n = n0 + mm;
      if (n < N && k < K)
        bv = widen(tb ? B[static_cast<size_t>(n) * ldb + k] : B[static_cast<size_t>(k) * ldb + n]);
      As[kk][mm] = av;
      Bs[kk][mm] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float& c = C[static_cast<size_t>(m) * ldc + n];
      c = beta == 0.f ? alpha * acc[i][j] : fmaf(beta, c, alpha * acc[i][j]);
    }
  }
}

}  // namespace
}  // namespace gsvk

using namespace gsvk;

extern "C" int gsvk_sgemm(char transa, char transb, int M, int N, int K, float alpha,
                          const float* A, int lda, const float* B, int ldb, float beta, float* C,
                          int ldc, gsvk_stream_t stream) {
  const int ta = (transa == 'T' || transa == 't'), tb = (transb == 'T' || transb == 't');
  if (!(ta || transa == 'N' || transa == 'n') || !(tb || transb == 'N' || transb == 'n'))
    return fail(GSVK_ERR_INVALID, "sgemm: trans flags must be 'N' or 'T'");
  if (M < 0 || N < 0 || K < 0 || !C || (K > 0 && (!A || !B)))
    return fail(GSVK_ERR_INVALID, "sgemm: bad sizes or null pointer");
  if (ldc < N || lda < (ta ? M : K) || ldb < (tb ? K : N))
    return fail(GSVK_ERR_INVALID, "sgemm: leading dimension too small");
  if (M == 0 || N == 0) return GSVK_OK;
  dim3 grid((unsigned)((N + kT - 1) / kT), (unsigned)((M + kT - 1) / kT));
  sgemm_kernel<float><<<grid, 256, 0, as_cuda(stream)>>>(M, N, K, alpha, A, lda, ta, B, ldb, tb,
                                                         beta, C, ldc);
  return check_launch("sgemm_kernel");
}

extern "C" int gsvk_gemm_nt_f16w(const float* x, size_t T, size_t in, const uint16_t* w,
                                 size_t out, float* y, gsvk_stream_t stream) {
  if (!x || !w || !y) return fail(GSVK_ERR_INVALID, "gemm_nt_f16w: null pointer");
  if (T > INT32_MAX || in > INT32_MAX || out > INT32_MAX)
    return fail(GSVK_ERR_INVALID, "gemm_nt_f16w: dimension beyond 2^31");
  if (T == 0 || out == 0) return GSVK_OK;
  const int M = (int)T, N = (int)out, K = (int)in;
  dim3 grid((unsigned)((N + kT - 1) / kT), (unsigned)((M + kT - 1) / kT));
  sgemm_kernel<uint16_t><<<grid, 256, 0, as_cuda(stream)>>>(M, N, K, 1.f, x, K, 0, w, K, 1, 0.f,
                                                            y, N);
  return check_launch("sgemm_kernel<f16 B>");
}
