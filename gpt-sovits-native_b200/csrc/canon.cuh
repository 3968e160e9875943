// canon.cuh — the canonical T2S arithmetic, reproduced bit for bit.
//
// The reference leaves the association of its sums to NEON register blocking
// (and Accelerate); the T2S path here fixes one order and evaluates it
// identically on the CPU oracle and on the device, so that greedy token
// streams are identical by construction, not by luck of the logit margins:
//   dot32     the gemv_fmlal.cpp:40-109 association: 32 accumulators (8 groups
//             x 4 lanes) over 64-element steps, low then high half of each
//             8-element slice; group sums (a0+a1)+(a2+a3); groups added in
//             order.  One accumulator per lane of a warp.
//   dot_kv    dot_f16kv (t2s_engine.cpp:69-99): 4 x 4 accumulators over
//             16-element steps, (a0+a1)+(a2+a3) per lane, (s0+s2)+(s1+s3).
//   ln_canon  kern.cpp:27-58: 8-lane fp32 sums, fp64 mean / biased variance.
//   exp_det   Cody-Waite reduction + degree-7 Taylor polynomial (within 2 ulp
//             of expf), used by the chunked softmax.
// Every multiply feeding an add that the order keeps separate is written with
// __fmul_rn / __fadd_rn so that the compiler cannot contract it into an FMA.
#pragma once

#include "common.cuh"

namespace gsvk {

__device__ __forceinline__ float exp_det(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = fmaf(n, -0.693359375f, x);
  r = fmaf(n, 2.12194440e-4f, r);
  float p = 1.98412698e-4f;
  p = fmaf(p, r, 1.38888889e-3f);
  p = fmaf(p, r, 8.33333333e-3f);
  p = fmaf(p, r, 4.16666667e-2f);
  p = fmaf(p, r, 1.66666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = static_cast<int>(n);
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// Canonical dot of an fp16 row with fp32 activations, one warp; every lane
// returns the same value.  w and x may live in shared or global memory.
__device__ __forceinline__ float warp_dot32(const uint16_t* w, const float* x, int n) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  const int vec_end = n & ~63;
  float acc = 0.f;
  if (n == 512) {  // the T2S width: every load ahead of the chain
    float wv[16], xv[16];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      wv[2 * b] = h2f(w[64 * b + o0]);
      wv[2 * b + 1] = h2f(w[64 * b + o0 + 4]);
      xv[2 * b] = x[64 * b + o0];
      xv[2 * b + 1] = x[64 * b + o0 + 4];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) acc = fmaf(wv[j], xv[j], acc);
  } else {
#pragma unroll 4
    for (int i = 0; i < vec_end; i += 64) {
      acc = fmaf(h2f(w[i + o0]), x[i + o0], acc);
      acc = fmaf(h2f(w[i + o0 + 4]), x[i + o0 + 4], acc);
    }
  }
  const float t = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  const float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
  float s = __shfl_sync(0xffffffffu, u, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, u, 4 * j));
  for (int i = vec_end; i < n; ++i) s = fmaf(h2f(w[i]), x[i], s);
  return s;
}

// Canonical q . k over HD dims by a 16-lane group (lanes g*16 .. g*16+15 of a
// warp); q_reg[c] holds q[16c + (lane & 15)].  Lane (lane & 15) == 0 of the
// group ends with the result (others hold partial combinations).
template <int HD>
__device__ __forceinline__ float group16_dot_kv(const float* q_reg, const uint16_t* krow) {
  const int L = threadIdx.x & 15;
  float a = 0.f;
#pragma unroll
  for (int c = 0; c < HD / 16; ++c) a = fmaf(q_reg[c], h2f(krow[16 * c + L]), a);
  const float t = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
  const float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 8));
  const float v = __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, 2));
  return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
}

// 1 / sqrt(v) rounded to float exactly as (float)(1.0 / sqrt(v)) with both
// double operations correctly rounded (kern.cpp:55).
//
// A float candidate r is accepted when y = 1/sqrt(v) lies strictly inside
// (m_lo, m_hi), the midpoints between r and its float neighbours, with a
// relative margin of at least 2^-48.  The test is exact: m has at most 25
// significant bits, so m*m is exact in double, and y < m <=> m^2 v > 1, whose
// sign one fused multiply-add m^2 v - 1 gives exactly (its value s is also
// accurate: (m - y) / y ~ s / 2).  The reference value (two correctly rounded
// double operations) lies within 2^-51 * y of y, so it rounds to r as well.
// The candidate is the float reciprocal square root refined by one Newton
// step in double (then almost always the nearest float, so one test
// suffices); a failed test moves it one ulp and tests again, and a y within
// the margin of a midpoint (about one call in 2^23), or a non-finite or zero
// candidate, takes the exact sqrt-then-divide path.  The test alone decides
// correctness: the candidate's accuracy only decides the speed.
__device__ __forceinline__ float rstd_f32(double v) {
  const double y0 = static_cast<double>(rsqrtf(__double2float_rn(v)));
  const double y1 = y0 * fma(-0.5 * v * y0, y0, 1.5);
  float r = __double2float_rn(y1);
#pragma unroll 1
  for (int step = 0; step < 3; ++step) {
    if (!(r > 0.0f) || isinf(r)) break;
    const int bits = __float_as_int(r);  // r positive and finite: neighbours by integer steps
    const double rd = static_cast<double>(r);
    const double mhi = 0.5 * (rd + static_cast<double>(__int_as_float(bits + 1)));
    const double mlo = 0.5 * (rd + static_cast<double>(__int_as_float(bits - 1)));
    const double shi = fma(mhi * mhi, v, -1.0);  // > 0  <=>  y < mhi
    const double slo = fma(mlo * mlo, v, -1.0);  // < 0  <=>  y > mlo
    if (shi > 0x1p-46 && slo < -0x1p-46) return r;
    if (shi <= 0.0)
      r = __int_as_float(bits + 1);
    else if (slo >= 0.0)
      r = __int_as_float(bits - 1);
    else
      break;  // y within the margin of a midpoint
  }
  return static_cast<float>(__ddiv_rn(1.0, __dsqrt_rn(v)));
}

// Sum chains of ln_canon for thread l (0..7: sum of x[l], x[l+8], ...;
// 8..15: the same chains of squares, fused multiply-add), element order.
template <int N>
__device__ __forceinline__ float ln_chain_fixed(const float* buf, int l, bool sq) {
  float v[N / 8];
#pragma unroll
  for (int u = 0; u < N / 8; ++u) v[u] = buf[l + 8 * u];
  float a = 0.f;
#pragma unroll
  for (int u = 0; u < N / 8; ++u) a = sq ? fmaf(v[u], v[u], a) : __fadd_rn(a, v[u]);
  return a;
}

// LayerNorm of n values held in shared memory `buf`, in place, whole block.
// scratch: >= 18 floats of shared memory.  Threads 0-7 run the 8 sum chains,
// 8-15 the 8 sum-of-squares chains (each in element order); thread 0 then
// forms mean / variance / rstd in fp64.  rounded (optional) receives
// f16-rounded copies of the outputs (the next GEMV's fp16 activations).
__device__ __forceinline__ void ln_canon(float* buf, const float* g, const float* b, int n,
                                         double eps, float* scratch, float* rounded = nullptr) {
  const int tid = threadIdx.x;
  const int vec_end = n & ~7;
  if (tid < 16) {
    const int l = tid & 7;
    const bool sq = tid >= 8;
    float a = 0.f;
    if (n == 512) {
      a = ln_chain_fixed<512>(buf, l, sq);
    } else {
      int i = l;
      for (; i + 56 < vec_end; i += 64) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = buf[i + 8 * u];
#pragma unroll
        for (int u = 0; u < 8; ++u) a = sq ? fmaf(v[u], v[u], a) : __fadd_rn(a, v[u]);
      }
      for (; i < vec_end; i += 8) {
        const float v = buf[i];
        a = sq ? fmaf(v, v, a) : __fadd_rn(a, v);
      }
    }
      // lanes 0-7 and 8-15 combine as ((0+1)+(2+3))+((4+5)+(6+7))
    float t = __fadd_rn(a, __shfl_xor_sync(0x0000ffffu, a, 1));
    t = __fadd_rn(t, __shfl_xor_sync(0x0000ffffu, t, 2));
    t = __fadd_rn(t, __shfl_xor_sync(0x0000ffffu, t, 4));
    const float qsum = __shfl_sync(0x0000ffffu, t, 8);
      if (tid == 0) {
      double sum = static_cast<double>(t), sqs = static_cast<double>(qsum);
      for (int i = vec_end; i < n; ++i) {
        const double xv = static_cast<double>(buf[i]);
        sum = __dadd_rn(sum, xv);
        sqs = __dadd_rn(sqs, __dmul_rn(xv, xv));
      }
      const double dn = static_cast<double>(n);
      // x / 2^k == x * 2^-k exactly: skip the fp64 divide for power-of-two n
      const bool pow2 = (n & (n - 1)) == 0;
      const double inv_n = pow2 ? 1.0 / dn : 0.0;
      const float mean = static_cast<float>(pow2 ? __dmul_rn(sum, inv_n) : __ddiv_rn(sum, dn));
      const double md = static_cast<double>(mean);
      const double ex2 = pow2 ? __dmul_rn(sqs, inv_n) : __ddiv_rn(sqs, dn);
      float var = static_cast<float>(__dsub_rn(ex2, __dmul_rn(md, md)));
      if (!(var >= 0.0f)) {
        double s2 = 0.0;
        for (int i = 0; i < n; ++i) {
          const double d = __dsub_rn(static_cast<double>(buf[i]), md);
          s2 = __dadd_rn(s2, __dmul_rn(d, d));
        }
        var = static_cast<float>(pow2 ? __dmul_rn(s2, inv_n) : __ddiv_rn(s2, dn));
      }
          scratch[16] = mean;
      scratch[17] = rstd_f32(__dadd_rn(static_cast<double>(var), eps));
        }
  }
  __syncthreads();
  const float mean = scratch[16], rstd = scratch[17];
  for (int i = tid; i < n; i += blockDim.x) {
    const float v = fmaf(__fmul_rn(__fsub_rn(buf[i], mean), rstd), g[i], b[i]);
    buf[i] = v;
    if (rounded) rounded[i] = h2f(f2h(v));
  }
  __syncthreads();
}

// ln_canon's mean and rstd computed by ONE warp (any warp; several warps may
// compute the same statistics concurrently): lanes (l & 15) run ln_canon's 16
// chains (lanes 16-31 repeat them), every lane then holds both sums and forms
// mean / variance / rstd itself in fp64.  Same values as ln_canon.
__device__ __forceinline__ void warp_ln_stats(const float* buf, int n, double eps, float* mean_out,
                                              float* rstd_out) {
  const int lane = threadIdx.x & 31;
  const int l = lane & 7;
  const bool sq = (lane & 8) != 0;
  const int vec_end = n & ~7;
  float a = 0.f;
  if (n == 512) {
    a = ln_chain_fixed<512>(buf, l, sq);
  } else {
    for (int i = l; i < vec_end; i += 8) {
      const float v = buf[i];
      a = sq ? fmaf(v, v, a) : __fadd_rn(a, v);
    }
  }
  // lanes 0-7 and 8-15 combine as ((0+1)+(2+3))+((4+5)+(6+7))
  float t = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
  t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
  t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
  const float ssum = __shfl_sync(0xffffffffu, t, 0);
  const float qsum = __shfl_sync(0xffffffffu, t, 8);
  double sum = static_cast<double>(ssum), sqs = static_cast<double>(qsum);
  for (int i = vec_end; i < n; ++i) {
    const double xv = static_cast<double>(buf[i]);
    sum = __dadd_rn(sum, xv);
    sqs = __dadd_rn(sqs, __dmul_rn(xv, xv));
  }
  const double dn = static_cast<double>(n);
  const bool pow2 = (n & (n - 1)) == 0;
  const double inv_n = pow2 ? 1.0 / dn : 0.0;
  const float mean = static_cast<float>(pow2 ? __dmul_rn(sum, inv_n) : __ddiv_rn(sum, dn));
  const double md = static_cast<double>(mean);
  const double ex2 = pow2 ? __dmul_rn(sqs, inv_n) : __ddiv_rn(sqs, dn);
  float var = static_cast<float>(__dsub_rn(ex2, __dmul_rn(md, md)));
  if (!(var >= 0.0f)) {
    double s2 = 0.0;
    for (int i = 0; i < n; ++i) {
      const double d = __dsub_rn(static_cast<double>(buf[i]), md);
      s2 = __dadd_rn(s2, __dmul_rn(d, d));
    }
    var = static_cast<float>(pow2 ? __dmul_rn(s2, inv_n) : __ddiv_rn(s2, dn));
  }
  *mean_out = mean;
  *rstd_out = rstd_f32(__dadd_rn(static_cast<double>(var), eps));
}

// One LayerNorm output element, ln_canon's arithmetic.
__device__ __forceinline__ float ln_val(float x, float mean, float rstd, float g, float b) {
  return fmaf(__fmul_rn(__fsub_rn(x, mean), rstd), g, b);
}

// This lane's 16 activations of the 512-wide canonical dot (xr[2b] = element
// 64b + o0, xr[2b + 1] = 64b + o0 + 4), optionally through a LayerNorm
// (mean, rstd, g, b) and/or rounded to fp16 values.
__device__ __forceinline__ void lane_act512(const float* x, bool ln, float mean, float rstd, const float* g,
                                            const float* b, bool round16, float* xr) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int i = 64 * (k >> 1) + o0 + 4 * (k & 1);
    float v = x[i];
    if (ln) v = ln_val(v, mean, rstd, g[i], b[i]);
    xr[k] = round16 ? h2f(f2h(v)) : v;
  }
}

// warp_dot32 (n = 512) with the activations in registers (lane_act512 layout).
__device__ __forceinline__ float warp_dot512_r(const uint16_t* w, const float* xr) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  float wv[16];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    wv[2 * b] = h2f(w[64 * b + o0]);
    wv[2 * b + 1] = h2f(w[64 * b + o0 + 4]);
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) acc = fmaf(wv[j], xr[j], acc);
  const float t = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  const float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
  float s = __shfl_sync(0xffffffffu, u, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, u, 4 * j));
  return s;
}

// fp32(a) * fp32(b) + c rounded once, a and b fp16 bits: the product of two
// fp16 values is exact in fp32, so this equals fmaf(h2f(a), h2f(b), c)
// without the two conversions (mixed-precision fma).
__device__ __forceinline__ float fma_hh(uint16_t a, uint16_t b, float c) {
  float d;
  asm("{\n\t.reg .f16 ha, hb;\n\tmov.b16 ha, %1;\n\tmov.b16 hb, %2;\n\t"
      "fma.rn.f32.f16 %0, ha, hb, %3;\n\t}"
      : "=f"(d)
      : "h"(a), "h"(b), "f"(c));
  return d;
}

// This lane's 16 activations (lane_act512 layout) as fp16 bits, rounded to
// nearest even from the fp32 values (optionally through a LayerNorm).
__device__ __forceinline__ void lane_act512_h(const float* x, bool ln, float mean, float rstd, const float* g,
                                              const float* b, uint16_t* xh) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
#pragma unroll
  for (int k = 0; k < 16; k += 2) {
    const int i = 64 * (k >> 1) + o0;
    float v0 = x[i], v1 = x[i + 4];
    if (ln) {
      v0 = ln_val(v0, mean, rstd, g[i], b[i]);
      v1 = ln_val(v1, mean, rstd, g[i + 4], b[i + 4]);
    }
    const uint32_t p = f2h2(v0, v1);  // one conversion for both
    xh[k] = static_cast<uint16_t>(p & 0xffffu);
    xh[k + 1] = static_cast<uint16_t>(p >> 16);
  }
}

// warp_dot512_r for fp16 activations xh (bits): the same chain and result.
__device__ __forceinline__ float warp_dot512_h(const uint16_t* w, const uint16_t* xh) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  uint16_t wv[16];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    wv[2 * b] = w[64 * b + o0];
    wv[2 * b + 1] = w[64 * b + o0 + 4];
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) acc = fma_hh(wv[j], xh[j], acc);
  const float t = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  const float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
  float s = __shfl_sync(0xffffffffu, u, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, u, 4 * j));
  return s;
}
__device__ __forceinline__ void warp_dot512x2_h(const uint16_t* w0, const uint16_t* w1, const uint16_t* xh,
                                                float* r0, float* r1) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  uint16_t u0[16], u1[16];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    u0[2 * b] = w0[64 * b + o0];
    u0[2 * b + 1] = w0[64 * b + o0 + 4];
    u1[2 * b] = w1[64 * b + o0];
    u1[2 * b + 1] = w1[64 * b + o0 + 4];
  }
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    a0 = fma_hh(u0[j], xh[j], a0);
    a1 = fma_hh(u1[j], xh[j], a1);
  }
  float t0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
  float t1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
  t0 = __fadd_rn(t0, __shfl_xor_sync(0xffffffffu, t0, 2));
  t1 = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 2));
  float s0 = __shfl_sync(0xffffffffu, t0, 0), s1 = __shfl_sync(0xffffffffu, t1, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) {
    s0 = __fadd_rn(s0, __shfl_sync(0xffffffffu, t0, 4 * j));
    s1 = __fadd_rn(s1, __shfl_sync(0xffffffffu, t1, 4 * j));
  }
  *r0 = s0;
  *r1 = s1;
}

// Two of them sharing the activations (chains interleaved).
__device__ __forceinline__ void warp_dot512x2_r(const uint16_t* w0, const uint16_t* w1, const float* xr,
                                                float* r0, float* r1) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  float u0[16], u1[16];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    u0[2 * b] = h2f(w0[64 * b + o0]);
    u0[2 * b + 1] = h2f(w0[64 * b + o0 + 4]);
    u1[2 * b] = h2f(w1[64 * b + o0]);
    u1[2 * b + 1] = h2f(w1[64 * b + o0 + 4]);
  }
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    a0 = fmaf(u0[j], xr[j], a0);
    a1 = fmaf(u1[j], xr[j], a1);
  }
  float t0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
  float t1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
  t0 = __fadd_rn(t0, __shfl_xor_sync(0xffffffffu, t0, 2));
  t1 = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 2));
  float s0 = __shfl_sync(0xffffffffu, t0, 0), s1 = __shfl_sync(0xffffffffu, t1, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) {
    s0 = __fadd_rn(s0, __shfl_sync(0xffffffffu, t0, 4 * j));
    s1 = __fadd_rn(s1, __shfl_sync(0xffffffffu, t1, 4 * j));
  }
  *r0 = s0;
  *r1 = s1;
}

// Two canonical dots sharing x (independent chains interleaved for ILP).
__device__ __forceinline__ void warp_dot32x2(const uint16_t* w0, const uint16_t* w1,
                                             const float* x, int n, float* r0, float* r1) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  const int vec_end = n & ~63;
  float a0 = 0.f, a1 = 0.f;
  if (n == 512) {  // the T2S width: every load ahead of the chains
    float u0[16], u1[16], xv[16];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      xv[2 * b] = x[64 * b + o0];
      xv[2 * b + 1] = x[64 * b + o0 + 4];
      u0[2 * b] = h2f(w0[64 * b + o0]);
      u0[2 * b + 1] = h2f(w0[64 * b + o0 + 4]);
      u1[2 * b] = h2f(w1[64 * b + o0]);
      u1[2 * b + 1] = h2f(w1[64 * b + o0 + 4]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      a0 = fmaf(u0[j], xv[j], a0);
      a1 = fmaf(u1[j], xv[j], a1);
    }
  } else {
#pragma unroll 4
    for (int i = 0; i < vec_end; i += 64) {
      const float xl = x[i + o0], xh = x[i + o0 + 4];
      a0 = fmaf(h2f(w0[i + o0]), xl, a0);
      a1 = fmaf(h2f(w1[i + o0]), xl, a1);
      a0 = fmaf(h2f(w0[i + o0 + 4]), xh, a0);
      a1 = fmaf(h2f(w1[i + o0 + 4]), xh, a1);
    }
  }
  float t0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
  float t1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
  t0 = __fadd_rn(t0, __shfl_xor_sync(0xffffffffu, t0, 2));
  t1 = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 2));
  float s0 = __shfl_sync(0xffffffffu, t0, 0), s1 = __shfl_sync(0xffffffffu, t1, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) {
    s0 = __fadd_rn(s0, __shfl_sync(0xffffffffu, t0, 4 * j));
    s1 = __fadd_rn(s1, __shfl_sync(0xffffffffu, t1, 4 * j));
  }
  for (int i = vec_end; i < n; ++i) {
    s0 = fmaf(h2f(w0[i]), x[i], s0);
    s1 = fmaf(h2f(w1[i]), x[i], s1);
  }
  *r0 = s0;
  *r1 = s1;
}

// Canonical q . k (dot_f16kv order) by ONE thread: 4 x 4 accumulators over
// 16-element steps, (a0+a1)+(a2+a3) per lane, then (s0+s2)+(s1+s3).
template <int HD>
__device__ __forceinline__ float thread_dot_kv(const float* q, const uint4* krow) {
  float a[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int l = 0; l < 4; ++l) a[j][l] = 0.f;
#pragma unroll
  for (int e = 0; e < HD; e += 16) {
    float kf[16];
    unpack8(krow[e / 8], kf);
    unpack8(krow[e / 8 + 1], kf + 8);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int l = 0; l < 4; ++l) a[j][l] = fmaf(q[e + 4 * j + l], kf[4 * j + l], a[j][l]);
  }
  float s[4];
#pragma unroll
  for (int l = 0; l < 4; ++l) s[l] = __fadd_rn(__fadd_rn(a[0][l], a[1][l]), __fadd_rn(a[2][l], a[3][l]));
  return __fadd_rn(__fadd_rn(s[0], s[2]), __fadd_rn(s[1], s[3]));
}

}  // namespace gsvk
