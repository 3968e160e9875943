// common.cuh — shared host/device helpers for the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gsvk.h"

namespace gsvk {

// ------------------------------------------------------------------ host side
// Records a printf-style message as the calling thread's last error and
// returns `code` (used as `return fail(GSVK_ERR_INVALID, "...")`).
int fail(int code, const char* fmt, ...);
// Converts a CUDA error into GSVK_ERR_CUDA with context; GSVK_OK otherwise.
int check_cuda(cudaError_t e, const char* what);
// cudaGetLastError after a launch.
int check_launch(const char* kernel);
// Device properties of the device current on the calling thread.
int sm_count();

inline cudaStream_t as_cuda(gsvk_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
// Launches `kernel` with a programmatic dependency on the previous kernel in
// `st` (it may start while that kernel drains; it must call griddep_wait()
// before reading that kernel's results).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               const char* name, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), name);
}
__host__ __device__ inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}
inline unsigned ceil_div(size_t a, size_t b) { return static_cast<unsigned>((a + b - 1) / b); }

// ---------------------------------------------------------------- device side
// Programmatic dependent launch.  griddep_wait() blocks until the kernels this
// launch depends on have completed and their writes are visible (a no-op when
// the launch carries no programmatic dependency); griddep_launch_dependents()
// lets the next kernel in the stream begin its independent prologue.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Aligns a dynamic shared-memory base to A bytes by pointer arithmetic on the
// shared array itself, so that the compiler keeps every access derived from
// it in the shared address space (a round trip through an integer would turn
// them all into generic loads and stores).
template <unsigned A>
__device__ __forceinline__ uint8_t* align_smem(uint8_t* base) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(base));
  return base + ((A - (a & (A - 1u))) & (A - 1u));
}
__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }
// Two fp32 -> packed fp16 pair (low half = a), RNE, one conversion instruction.
__device__ __forceinline__ uint32_t f2h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Streaming 128-bit load that bypasses L1 allocation (weights are read once
// per launch; keeping them out of L1 leaves it to the reused activations).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 8 packed fp16 (one uint4) -> 8 fp32.
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Maximum over the full warp in one instruction (sm_100a's floating-point
// redux): exact, the value a butterfly of fmaxf would give.
__device__ __forceinline__ float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// Epilogue activation (GSVK_ACT_*), the reference's expressions:
// relu kern.cpp:85, gelu_erf bert_ops.hpp:25, leaky nn_ops.hpp:48,
// tanh dec.hpp:344.
//
// GELU(x) = 0.5 x (1 + erf(x / sqrt 2)) = x Phi(x).  With u = min(|x|, 5.5),
//   Phi(-u) = 2^(h(u) - u^2 log2(e) / 2),
// h a degree-10 polynomial least-squares fitted (double precision, 6000
// Chebyshev nodes on [0, 5.5]) to log2 Phi(-u) + u^2 log2(e) / 2, a smooth
// function of u; Phi(x) = 1 - Phi(-u) for x >= 0, Phi(-u) otherwise, so the
// negative tail keeps its relative accuracy.  One ex2, 14 FMA-pipe and 3
// ALU operations.  Evaluated in fp32 over [-9, 9]: within 3.9e-7 of the exact
// x Phi(x) (under one ulp of the result) and within 2.4e-6 relative where
// |GELU(x)| > 1e-6.  The clamp leaves the exact -x^2 term, so past
// |x| = 5.5 it only perturbs values smaller than 1.1e-7.
__device__ __forceinline__ float gelu_erf(float x) {
  const float u = fminf(fabsf(x), 5.5f);
  float h = -1.725302567e-08f;
  h = fmaf(h, u, 5.477549507e-07f);
  h = fmaf(h, u, -7.458289474e-06f);
  h = fmaf(h, u, 5.484473149e-05f);
  h = fmaf(h, u, -2.005067072e-04f);
  h = fmaf(h, u, -1.761470485e-04f);
  h = fmaf(h, u, 7.180649787e-03f);
  h = fmaf(h, u, -5.261564627e-02f);
  h = fmaf(h, u, 2.621913850e-01f);
  h = fmaf(h, u, -1.151113272e+00f);
  h = fmaf(h, u, -9.999998212e-01f);
  float q;  // Phi(-|x|)
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(q) : "f"(fmaf(-0.721347520444f, x * x, h)));
  return x * (x >= 0.f ? 1.f - q : q);
}
// tanh stays out of line: epilogues unroll apply_act per element, and
// inlining tanhf into every copy makes those loops overflow the
// instruction cache (it only runs in the decoder's last conv).
static __device__ __noinline__ float apply_act_transcendental(float v, int act) {
  return act == GSVK_ACT_GELU_ERF ? gelu_erf(v) : tanhf(v);
}
__device__ __forceinline__ float apply_act(float v, int act, float slope) {
  switch (act) {
    case GSVK_ACT_RELU: return v > 0.f ? v : 0.f;
    case GSVK_ACT_LEAKY: return v < 0.f ? v * slope : v;
    case GSVK_ACT_GELU_ERF: return gelu_erf(v);
    case GSVK_ACT_TANH: return apply_act_transcendental(v, act);
    default: return v;
  }
}

// Activation over a small register array with the dispatch hoisted out of
// the element loop (keeps unrolled epilogue bodies small).
template <int NV>
__device__ __forceinline__ void act_array(float* v, int act, float slope) {
  switch (act) {
    case GSVK_ACT_NONE: break;
    case GSVK_ACT_RELU:
#pragma unroll
      for (int j = 0; j < NV; ++j) v[j] = v[j] > 0.f ? v[j] : 0.f;
      break;
    case GSVK_ACT_LEAKY:
#pragma unroll
      for (int j = 0; j < NV; ++j) v[j] = v[j] < 0.f ? v[j] * slope : v[j];
      break;
    case GSVK_ACT_GELU_ERF:
#pragma unroll
      for (int j = 0; j < NV; ++j) v[j] = gelu_erf(v[j]);
      break;
    default:
      for (int j = 0; j < NV; ++j) v[j] = apply_act_transcendental(v[j], act);
  }
}

}  // namespace gsvk
