// gsvk_internal.hpp — declarations shared between the library's translation
// units (not part of the public ABI).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace gsvk {

// Per-device status word written by bounded device-side waits (DEV_TIMEOUT).
uint32_t* device_status();

// K-major (row-major [rows, kc], leading dimension ld elements) fp16 tensor
// map with a box of bk x box_rows and the swizzle matching bk.
int make_kmajor_map(CUtensorMap* map, const uint16_t* base, long long rows, long long kc,
                    long long ld, int box_rows, int bk);
int tc_pick_bn(long long M, long long N);
// Launches the tensor-core kernel for problem p (bn = 0 picks the tile width).
// a_cols / b_cols: width of the A / B tensor maps when problems address
// column windows of a wider matrix (batched mode); 0 = p.kc.
int tc_run(const uint16_t* a, long long a_rows, long long lda, const uint16_t* b,
           long long b_rows, long long ldb, TcProblem p, const TcEpilogue& e, int bn,
           cudaStream_t st, long long a_cols = 0, long long b_cols = 0);
TcEpilogue make_epilogue();
// Split-K cluster GEMM for few-row activations (gemm_skinny.cu):
// C[m, n] = epi(sum_k x[m, k] w[n, k]) for M <= 128; pdl = launch with a
// programmatic dependency on the previous kernel in the stream; force_split
// (a power of two <= 8) overrides the K split chosen from the shape.
bool skinny_fits(long long M, long long N, long long K, long long ldx, long long ldw,
                 const void* x, const void* w);
int skinny_run(const uint16_t* x, int M, long long ldx, const uint16_t* w, int N, long long ldw,
               int K, const TcEpilogue& e, cudaStream_t st, bool pdl, int force_split = 0);
// The gsvk_gemm_f16_ex dispatch.  static_b: B is registered weights, never
// written by device work (the launch is then a programmatic dependent of the
// previous kernel, whose set-up and first B loads overlap that kernel's end).
int gemm_ex_run(const gsvk_gemm_args* g, cudaStream_t st, bool static_b);
// CUDA-core fallback for shapes the TMA path cannot express (K or leading
// dimensions not multiples of 8, unaligned bases).
int simt_gemm(const gsvk_gemm_args* g, const TcEpilogue& e, cudaStream_t st);
int gemv_ex(const uint16_t* w, const void* x, int x_is_f16, float* y, uint16_t* yh, size_t out,
            size_t in, const float* bias, const float* residual, int act, float slope,
            cudaStream_t st);

}  // namespace gsvk
