// gemm_tc.cuh — warp-specialised persistent tensor-core GEMM for sm_100a.
//
//   C[row(i), n] = epi( sum_{t < taps} sum_k A[i + a_shift(t), k] * B[b_row(t) + n, k] )
//
// A (activations) and B (weights) are fp16, K-major (row-major [rows, K]),
// fetched by TMA into swizzled shared-memory stages; tcgen05.mma
// (cta_group::1, kind::f16, M = 128, N = BN, K = 16) accumulates fp32 in TMEM;
// the epilogue warps read TMEM with tcgen05.ld and apply bias / activation /
// residual before storing fp32 and/or fp16.
//
// The "taps" loop turns the same mainloop into:
//   plain GEMM          taps = 1, a_shift = 0, b_row = 0
//   conv1d (implicit)   tap t: a_shift = t*dil - pad, b_row = t*Co   (A = x[T, Ci] channels-last,
//                        B = W[k][Co][Ci]); rows outside [0, T) come back as zeros from TMA
//   ConvTranspose1d     phase r, tap m: a_shift = -m, b_row = (r + m*u)*Co,
//                        output row = q*u + r - pad with q = i + q0(r)   (polyphase, no scatter)
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer and TMEM
// owner, warps 2..9 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).  For
// tiles wider than 64 columns warps 2..5 take the left half of the columns
// and 6..9 the right half (two TMEM accumulators); for narrower tiles the two
// groups take alternate tiles (four accumulators).  Bias and residual chunks
// are fetched one chunk ahead of their use.
// Several TMEM accumulators let the epilogue of tile i overlap the mainloop of
// the following tiles.  Every mbarrier wait is bounded (see tma.cuh).
#pragma once

#include "tma.cuh"

namespace gsvk {

struct TcEpilogue {
  const float* bias;      // [N] or null
  const float* residual;  // fp32 [rows, ld_res] at the output row, or null
  float* c32;             // fp32 output or null
  uint16_t* c16;          // fp16 output or null
  uint16_t* c16_act;      // optional second fp16 output = act2(value)
  long long ld_c32, ld_c16, ld_res, ld_c16_act;
  int act;                // applied to alpha*acc + bias, before the residual add
  float slope;
  int act2;               // activation for c16_act
  float slope2;
  float alpha;
  float res_scale;        // y = act(alpha*acc + bias) + res_scale * residual
  // Optional transposed output of the columns >= vt_c0 (the V block of a
  // fused QKV projection): column vt_c0 + h*vt_dh + d of row b*vt_T + t goes
  // to vt[((b*vt_H + h)*vt_dh + d)*vt_ld + t] as fp16, and those columns
  // skip the other outputs.
  uint16_t* vt;
  long long vt_ld;
  int vt_c0, vt_T, vt_dh, vt_H;
  // Optional running mean (the average over the multi-receptive-field
  // residual blocks): with mean_sum set, the value y above contributes
  // t = y * mean_scale, s = mean_first ? t : mean_sum + t is stored back to
  // mean_sum (same [rows, ld_c32] layout as c32), and the outputs written
  // after it receive s in place of y (c32 / c16 = s, c16_act = act2(s)).
  float* mean_sum;
  float mean_scale;
  int mean_first;
};

struct TcProblem {
  int M;            // tile-space rows (per phase)
  int N;            // output columns
  int kc;           // K per tap
  int bk;           // K elements per stage: 16, 32 or 64 (swizzle 32/64/128 B)
  int taps;         // conv taps (plain GEMM: 1)
  int dil, pad;     // conv: a_shift(t) = t*dil - pad
  int b_tap_rows;   // rows of B per tap (Co)
  int convt;        // 1: ConvTranspose1d polyphase mode (taps = kernel k, dil = u)
  int phases;       // ConvT: u phases; batched: batch * bh; otherwise 1
  int out_rows;     // valid output rows (ConvT: T*u; others: M)
  // Batched mode (bh > 0, convt == 0): phase p = (b, h) with b = p / bh,
  // h = p % bh solves an independent GEMM whose operands and output start at
  //   A row b*a_rb + h*a_rh, A column h*a_ch;  B row b*b_rb + h*b_rh,
  //   B column h*b_ch;  output row b*c_rb + h*c_rh, output column h*c_ch.
  // (multi-head attention over a fused QKV buffer: one launch per product)
  // (plus constant column offsets a_c0 / b_c0, e.g. the K block of QKV)
  int bh;
  int a_rb, a_rh, a_ch, b_rb, b_rh, b_ch, c_rb, c_rh, c_ch;
  int a_c0, b_c0;
  // Window mode (win > 0, plain conv with one K block per tap and one column
  // tile): one TMA load of win = 128 + (taps-1)*dil input rows per output tile
  // serves every tap as a row-shifted operand descriptor (the swizzle follows
  // absolute shared-memory addresses, so any row start is valid); all taps'
  // weights are loaded once per CTA.
  int win;
  // Launched as a programmatic dependent of the previous kernel in the
  // stream: barrier set-up, TMEM allocation and (window mode) the weight
  // loads overlap that kernel's tail, so B must not be written by the
  // kernels this launch waits on.
  int pdl;
  // Two-SM kernel only: 0 = per-lane row stores; 1 = the fp16 output (c16)
  // and 2 = the fp32 output (c32, its fp32 residual loaded the same way) go
  // through swizzled shared-memory tiles and TMA bulk copies.
  int tma_epi;
  // One-SM kernel: 1 = the fp32 / running-mean / fp16 / activated-fp16 outputs leave through
  // swizzled shared-memory tiles (32 rows x 16 columns per warp) and TMA bulk
  // stores (plain and conv problems: contiguous output rows).
  int bulk_epi;
};

}  // namespace gsvk
