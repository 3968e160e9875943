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
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Epilogue activation (GSVK_ACT_*), the reference's expressions:
// relu kern.cpp:85, gelu_erf bert_ops.hpp:25 (its erf evaluated by the
// approximation below, within 1.5e-7), leaky nn_ops.hpp:48, tanh dec.hpp:344.
// erf(x) by Abramowitz & Stegun, Handbook of Mathematical Functions (1964),
// eq. 7.1.26 (Hastings' approximation): for x >= 0,
//   erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-x^2),
//   t = 1 / (1 + p x),  |error| <= 1.5e-7;  erf(-x) = -erf(x).
// Short enough to inline into unrolled epilogues.
__device__ __forceinline__ float erf_as7126(float x) {
  const float ax = fabsf(x);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, ax, 1.0f));  // approximate reciprocal (2 ulp)
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  const float y = fmaf(-poly * t, __expf(-ax * ax), 1.0f);
  return copysignf(y, x);
}
__device__ __forceinline__ float gelu_erf(float v) {
  return 0.5f * v * (1.f + erf_as7126(v * 0.70710678118654752440f));
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
