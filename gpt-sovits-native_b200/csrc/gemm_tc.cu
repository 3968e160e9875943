// gemm_tc.cu — tcgen05 / TMA tensor-core GEMM (see gemm_tc.cuh for the
// algorithm and roles) and its C-ABI entry points:
//   gsvk_gemm_f16 / gsvk_gemm_f16_ex      (kern::gemm_f16x_fmlal, accel::DenseF16 view)
//   gsvk_conv1d_f16 / gsvk_convt1d_f16    (sovits::Conv1d / ConvT1d as implicit GEMM)
#include <algorithm>

#include "gemm_tc.cuh"
#include "gsvk_internal.hpp"

namespace gsvk {

namespace {

constexpr int kBM = 128;
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quadrant, each half of the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemBudget = 200 * 1024;

struct TapPlan {
  int ntaps, q0, qmax, a_mul, a_off, b_first, b_step, o_mul, o_off;
  int a_row0, a_col0, b_row0, b_col0, c_row0, c_col0;  // batched-mode offsets
};

__device__ __forceinline__ TapPlan plan_for(const TcProblem& p, int phase) {
  TapPlan t;
  if (!p.convt) {
    t.ntaps = p.taps;
    t.q0 = 0;
    t.qmax = p.M - 1;
    t.a_mul = p.dil;
    t.a_off = -p.pad;
    t.b_first = 0;
    t.b_step = 1;
    t.o_mul = 1;
    t.o_off = 0;
    if (p.bh > 0) {
      const int b = phase / p.bh, h = phase - (phase / p.bh) * p.bh;
      t.a_row0 = b * p.a_rb + h * p.a_rh;
      t.a_col0 = p.a_c0 + h * p.a_ch;
      t.b_row0 = b * p.b_rb + h * p.b_rh;
      t.b_col0 = p.b_c0 + h * p.b_ch;
      t.c_row0 = b * p.c_rb + h * p.c_rh;
      t.c_col0 = h * p.c_ch;
    } else {
      t.a_row0 = t.a_col0 = t.b_row0 = t.b_col0 = t.c_row0 = t.c_col0 = 0;
    }
  } else {
    const int u = p.dil, k = p.taps, r = phase;
    t.ntaps = (k - r + u - 1) / u;
    const int num = p.pad - r;
    t.q0 = num > 0 ? (num + u - 1) / u : 0;
    const int top = p.out_rows - 1 + p.pad - r;
    t.qmax = top >= 0 ? top / u : -1;
    t.a_mul = -1;
    t.a_off = 0;
    t.b_first = r;
    t.b_step = u;
    t.o_mul = u;
    t.o_off = r - p.pad;
    t.a_row0 = t.a_col0 = t.b_row0 = t.b_col0 = t.c_row0 = t.c_col0 = 0;
  }
  return t;
}

// Bias and residual of one 16-column chunk, fetched one chunk ahead of its
// use (loads stay in flight: values are assigned under branches, never
// selected, so nothing waits for them until store16 consumes them).
__device__ __forceinline__ void load16(const float* src, bool full, int n0, int N, float* out) {
  if (full && aligned16(src)) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(src + j);
      out[j] = v.x;
      out[j + 1] = v.y;
      out[j + 2] = v.z;
      out[j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (n0 + j < N) out[j] = src[j];
  }
}

__device__ __forceinline__ void fetch16(const TcEpilogue& e, bool row_ok, long long orow, int n0,
                                        int N, int oc, bool bias_vec, float* bb, float* rr,
                                        float* ss) {
  const bool full = (n0 + 16 <= N);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    bb[j] = 0.f;
    rr[j] = 0.f;
    ss[j] = 0.f;
  }
  if (e.bias) {
    if (full && bias_vec) {
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(e.bias + n0 + j));
        bb[j] = v.x;
        bb[j + 1] = v.y;
        bb[j + 2] = v.z;
        bb[j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) bb[j] = __ldg(e.bias + n0 + j);
    }
  }
  if (e.residual && row_ok) load16(e.residual + orow * e.ld_res + oc + n0, full, n0, N, rr);
  if (e.mean_sum && !e.mean_first && row_ok)
    load16(e.mean_sum + orow * e.ld_c32 + oc + n0, full, n0, N, ss);
}

// n0: column within the problem (bias index, N bound); oc: output column
// offset (batched mode), added to n0 for the output and residual addresses.
// bb / rr / ss: this chunk's bias, residual and running-mean sum (from fetch16).
__device__ __forceinline__ void store16(const TcEpilogue& e, long long orow, int n0, int N,
                                        const uint32_t* r, int oc, const float* bb,
                                        const float* rr, const float* ss) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = fmaf(__uint_as_float(r[j]), e.alpha, bb[j]);
  const bool full = (n0 + 16 <= N);
  act_array<16>(v, e.act, e.slope);
  if (e.residual) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = fmaf(e.res_scale, rr[j], v[j]);
  }
  if (e.vt && n0 >= e.vt_c0) {  // V columns: transposed per (utterance, head)
    const long long b = orow / e.vt_T, t = orow - b * e.vt_T;
    const int col = n0 - e.vt_c0, hh = col / e.vt_dh, d0 = col - (col / e.vt_dh) * e.vt_dh;
    uint16_t* dst = e.vt + ((b * e.vt_H + hh) * e.vt_dh + d0) * e.vt_ld + t;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (full || n0 + j < N) dst[j * e.vt_ld] = f2h(v[j]);
    return;
  }
  if (e.mean_sum) {  // running mean: rounded multiply, then rounded add (no contraction)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float t = __fmul_rn(v[j], e.mean_scale);
      v[j] = e.mean_first ? t : __fadd_rn(ss[j], t);
    }
    float* dst = e.mean_sum + orow * e.ld_c32 + oc + n0;
    if (full && aligned16(dst)) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) dst[j] = v[j];
    }
  }
  if (e.c32) {
    float* dst = e.c32 + orow * e.ld_c32 + oc + n0;
    if (full && aligned16(dst)) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) dst[j] = v[j];
    }
  }
  if (e.c16) {
    uint16_t* dst = e.c16 + orow * e.ld_c16 + oc + n0;
    if (full && aligned16(dst)) {
      uint32_t pk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pk[j] = f2h2(v[2 * j], v[2 * j + 1]);
      reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    } else {
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) dst[j] = f2h(v[j]);
    }
  }
  if (e.c16_act) {
    act_array<16>(v, e.act2, e.slope2);
    uint16_t* dst = e.c16_act + orow * e.ld_c16_act + oc + n0;
    if (full && aligned16(dst)) {
      uint32_t pk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pk[j] = f2h2(v[2 * j], v[2 * j + 1]);
      reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    } else {
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) dst[j] = f2h(v[j]);
    }
  }
}

// Bulk-copy epilogue of the one-SM kernel: per epilogue warp two 4 KB
// buffers, each [fp32 32 x 16 | fp16 32 x 16 | activated fp16 32 x 16]; the
// fp32 tile has 64-byte rows in the 64-byte swizzle (16-byte unit j of row r
// at j ^ ((r >> 1) & 3)), the fp16 tiles 32-byte rows in the 32-byte swizzle
// (unit j at j ^ ((r >> 2) & 1)): a lane writing its own row hits eight
// distinct bank groups per eight lanes.
constexpr uint32_t kBulkBuf = 4096;
constexpr size_t kBulkStgBytes = static_cast<size_t>(kEpiWarps) * 2 * kBulkBuf;
__device__ __forceinline__ uint8_t* sw64_unit(uint8_t* t, int r, int j) {
  return t + r * 64 + ((j ^ ((r >> 1) & 3)) << 4);
}
__device__ __forceinline__ uint8_t* sw32_unit(uint8_t* t, int r, int j) {
  return t + r * 32 + ((j ^ ((r >> 2) & 1)) << 4);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO32, const __grid_constant__ CUtensorMap tmO16,
                   const __grid_constant__ CUtensorMap tmO16a,
                   const __grid_constant__ CUtensorMap tmMean, const TcProblem prob,
                   const TcEpilogue epi, int stages, uint32_t* status) {
  // Register copies of the parameter structs (see gemm_skinny.cu: references
  // into parameter space are re-read after every global store).
  const TcProblem p = prob;
  const TcEpilogue e = epi;
  // Narrow tiles (BN <= 64) have short, latency-bound epilogues: two groups of
  // four epilogue warps take alternate tiles (each its tile's every column)
  // and four TMEM accumulators let the MMAs run ahead.  Wide tiles: one group
  // splitting the columns, two accumulators.
  constexpr int kGroups = BN <= 64 ? 2 : 1;
  constexpr int kAcc = BN <= 64 ? 4 : 2;
  constexpr uint32_t kTmemCols = kAcc * BN <= 32 ? 32u : (kAcc * BN <= 64 ? 64u :
                                 (kAcc * BN <= 128 ? 128u : (kAcc * BN <= 256 ? 256u : 512u)));
  const int bk = p.bk;
  const uint32_t swz_bytes = static_cast<uint32_t>(bk) * 2;          // 32, 64 or 128
  const uint32_t swz_code = swz_bytes == 128 ? 2u : (swz_bytes == 64 ? 4u : 6u);
  const bool win = p.win > 0;
  // stage sizes: a tap tile, or (window mode) a whole input window rounded to the 1 KB swizzle atom
  const uint32_t a_bytes = win ? (static_cast<uint32_t>(p.win) * swz_bytes + 1023u) & ~1023u
                               : kBM * swz_bytes;
  const uint32_t b_bytes = BN * swz_bytes;
  const uint32_t b_region = win ? static_cast<uint32_t>(p.taps) * b_bytes
                                : static_cast<uint32_t>(stages) * b_bytes;
  const uint32_t sbo = 8 * swz_bytes;                                  // 8-row atom stride
  const int ksteps = bk / 16;
  constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + static_cast<size_t>(stages) * a_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + b_region);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + kAcc;
  uint64_t* bbar = tempty + kAcc;  // window mode: all taps' weights landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bbar + 1);
  uint8_t* bulk_stg = reinterpret_cast<uint8_t*>(  // bulk-copy epilogue buffers, 1 KB aligned
      (reinterpret_cast<uintptr_t>(bbar + 2) + 1023) & ~static_cast<uintptr_t>(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (p.M + kBM - 1) / kBM, n_tiles = (p.N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles * p.phases;
  const int kpt = (p.kc + bk - 1) / bk;  // k-blocks per tap

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps / kGroups);
    }
    mbar_init(bbar, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.bulk_epi) {
      if (e.c32) prefetch_tmap(&tmO32);
      if (e.c16) prefetch_tmap(&tmO16);
      if (e.c16_act) prefetch_tmap(&tmO16a);
      if (e.mean_sum) prefetch_tmap(&tmMean);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Programmatic dependent launch: everything above, and the weight loads of
  // window mode, overlap the previous kernel; every access to activations and
  // outputs comes after griddep_wait (a no-op for an ordinary launch).
  const bool b_early = win && p.pdl;
  if (b_early && threadIdx.x == 0) {
    mbar_arrive_expect_tx(bbar, b_region);
    for (int t = 0; t < p.taps; ++t)
      tma_load_2d(sB + static_cast<size_t>(t) * b_bytes, &tmB, bbar, 0, t * p.b_tap_rows);
  }
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int it = 0;
      bool ok = true;
      if (win) {
        // every tap's weights once; then one input window per tile
        if (!b_early) {
          mbar_arrive_expect_tx(bbar, b_region);
          for (int t = 0; t < p.taps; ++t)
            tma_load_2d(sB + static_cast<size_t>(t) * b_bytes, &tmB, bbar, 0, t * p.b_tap_rows);
        }
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
          const int mt = tile;  // one column tile, one phase
          const int s = it % stages;
          const uint32_t ph = static_cast<uint32_t>(it / stages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(p.win) * swz_bytes);
          tma_load_2d(sA + static_cast<size_t>(s) * a_bytes, &tmA, &full[s], 0, mt * kBM - p.pad);
        }
      }
      for (int tile = blockIdx.x; tile < tiles && ok && !win; tile += gridDim.x) {
        const int phase = tile / (m_tiles * n_tiles);
        const int rem = tile - phase * m_tiles * n_tiles;
        const int mt = rem / n_tiles, nt = rem - (rem / n_tiles) * n_tiles;
        const TapPlan tp = plan_for(p, phase);
        for (int t = 0; t < tp.ntaps && ok; ++t) {
          const int a_row = tp.q0 + mt * kBM + tp.a_mul * t + tp.a_off + tp.a_row0;
          const int b_row = (tp.b_first + tp.b_step * t) * p.b_tap_rows + nt * BN + tp.b_row0;
          for (int kb = 0; kb < kpt; ++kb, ++it) {
            const int s = it % stages;
            const uint32_t ph = static_cast<uint32_t>(it / stages) & 1u;
            if (!mbar_wait(&empty[s], ph ^ 1u, status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
            tma_load_2d(sA + static_cast<size_t>(s) * a_bytes, &tmA, &full[s], kb * bk + tp.a_col0,
                        a_row);
            tma_load_2d(sB + static_cast<size_t>(s) * b_bytes, &tmB, &full[s], kb * bk + tp.b_col0,
                        b_row);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------------- MMA issuer
      int it = 0, tl = 0;
      bool ok = !win || mbar_wait(bbar, 0, status);
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++tl) {
        const int phase = tile / (m_tiles * n_tiles);
        const TapPlan tp = plan_for(p, phase);
        const int acc = tl % kAcc;
        const uint32_t aph = static_cast<uint32_t>(tl / kAcc) & 1u;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
        if (win) {
          // tap t reads window rows [t*dil, t*dil + 128): a start-address shift
          const int s = it % stages;
          const uint32_t ph = static_cast<uint32_t>(it / stages) & 1u;
          if (!mbar_wait(&full[s], ph, status)) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + static_cast<size_t>(s) * a_bytes);
          const uint32_t b_base = smem_u32(sB);
          for (int t = 0; t < p.taps; ++t) {
            const uint32_t a_t = a_base + static_cast<uint32_t>(t * p.dil) * swz_bytes;
            const uint32_t b_t = b_base + static_cast<uint32_t>(t) * b_bytes;
            for (int j = 0; j < ksteps; ++j)
              tc_mma_f16(d_tmem, smem_desc(a_t + 32u * j, sbo, swz_code),
                         smem_desc(b_t + 32u * j, sbo, swz_code), idesc, (t | j) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          ++it;
          tc_commit(&tfull[acc]);
          continue;
        }
        const int nk = tp.ntaps * kpt;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % stages;
          const uint32_t ph = static_cast<uint32_t>(it / stages) & 1u;
          if (!mbar_wait(&full[s], ph, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + static_cast<size_t>(s) * a_bytes);
          const uint32_t b_base = smem_u32(sB + static_cast<size_t>(s) * b_bytes);
          for (int j = 0; j < ksteps; ++j) {
            const uint64_t ad = smem_desc(a_base + 32u * j, sbo, swz_code);
            const uint64_t bd = smem_desc(b_base + 32u * j, sbo, swz_code);
            tc_mma_f16(d_tmem, ad, bd, idesc, (kk | j) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;            // TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;        // epilogue group (two groups) or column half
    const int cw = kGroups == 2 ? BN : BN / 2;  // columns per warp
    const int cbeg = kGroups == 2 ? 0 : half * cw;
    const bool cols_ok = true;
    const bool bias_vec = e.bias && aligned16(e.bias);
    int bulk_n = 0;  // bulk-copy epilogue chunks issued by this warp
    int tl = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tl) {
      if (kGroups == 2 && (tl & 1) != half) continue;  // the other group's tile
      const int phase = tile / (m_tiles * n_tiles);
      const int rem = tile - phase * m_tiles * n_tiles;
      const int mt = rem / n_tiles, nt = rem - (rem / n_tiles) * n_tiles;
      const TapPlan tp = plan_for(p, phase);
      const int acc = tl % kAcc;
      const uint32_t aph = static_cast<uint32_t>(tl / kAcc) & 1u;
      const int i = mt * kBM + quarter * 32 + lane;
      const int q = tp.q0 + i;
      const bool row_ok = (i < p.M) && (q <= tp.qmax);
      const long long orow = static_cast<long long>(q) * tp.o_mul + tp.o_off + tp.c_row0;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      float bnext[16], rnext[16], snext[16];
      fetch16(e, row_ok, orow, nt * BN + cbeg, p.N, tp.c_col0, bias_vec, bnext, rnext, snext);
      if (!mbar_wait(&tfull[acc], aph, status)) break;
      tc_fence_after();
      if (p.bulk_epi) {
        // bulk-copy epilogue: the per-row arithmetic of store16, results staged
        // in this warp's swizzled tiles, one bulk group per 16-column chunk
        const int row0 = mt * kBM + quarter * 32;
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + cw; c0 += 16) {
          if (nt * BN + c0 >= p.N) break;
          float bcur[16], rcur[16], scur[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            bcur[j] = bnext[j];
            rcur[j] = rnext[j];
            scur[j] = snext[j];
          }
          if (c0 + 16 < cbeg + cw)
            fetch16(e, row_ok, orow, nt * BN + c0 + 16, p.N, tp.c_col0, bias_vec, bnext, rnext,
                    snext);
          uint32_t r[16];
          tmem_ld16(t_row + static_cast<uint32_t>(c0), r);
          uint8_t* buf = bulk_stg + (static_cast<size_t>(warp - 2) * 2 + (bulk_n & 1)) * kBulkBuf;
          if (lane == 0) bulk_wait_read<1>();  // the store issued from `buf` has read it
          __syncwarp();
          tmem_ld_wait();
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = fmaf(__uint_as_float(r[j]), e.alpha, bcur[j]);
          act_array<16>(v, e.act, e.slope);
          if (e.residual) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = fmaf(e.res_scale, rcur[j], v[j]);
          }
          if (e.mean_sum) {  // running mean: rounded multiply, then rounded add (no contraction)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float t = __fmul_rn(v[j], e.mean_scale);
              v[j] = e.mean_first ? t : __fadd_rn(scur[j], t);
            }
          }
          if (e.c32 || e.mean_sum) {  // one fp32 tile serves both (the same values)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              *reinterpret_cast<float4*>(sw64_unit(buf, lane, k)) =
                  make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          }
          if (e.c16) {
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) pk[j] = f2h2(v[2 * j], v[2 * j + 1]);
            *reinterpret_cast<uint4*>(sw32_unit(buf + 2048, lane, 0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(sw32_unit(buf + 2048, lane, 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
          if (e.c16_act) {
            act_array<16>(v, e.act2, e.slope2);
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) pk[j] = f2h2(v[2 * j], v[2 * j + 1]);
            *reinterpret_cast<uint4*>(sw32_unit(buf + 3072, lane, 0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(sw32_unit(buf + 3072, lane, 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) {
            const int x = nt * BN + c0;
            if (e.mean_sum) tma_store_2d(&tmMean, buf, x, row0);
            if (e.c32) tma_store_2d(&tmO32, buf, x, row0);
            if (e.c16) tma_store_2d(&tmO16, buf + 2048, x, row0);
            if (e.c16_act) tma_store_2d(&tmO16a, buf + 3072, x, row0);
            bulk_commit();
          }
          ++bulk_n;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        continue;
      }
#pragma unroll 1
      for (int c0 = cbeg; c0 < cbeg + cw && cols_ok; c0 += 16) {
        float bcur[16], rcur[16], scur[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          bcur[j] = bnext[j];
          rcur[j] = rnext[j];
          scur[j] = snext[j];
        }
        if (c0 + 16 < cbeg + cw)
          fetch16(e, row_ok, orow, nt * BN + c0 + 16, p.N, tp.c_col0, bias_vec, bnext, rnext,
                  snext);
        uint32_t r[16];
        tmem_ld16(t_row + static_cast<uint32_t>(c0), r);
        tmem_ld_wait();
        if (row_ok && nt * BN + c0 < p.N)
          store16(e, orow, nt * BN + c0, p.N, r, tp.c_col0, bcur, rcur, scur);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (p.bulk_epi && lane == 0) bulk_wait<0>();  // every bulk store of this warp written
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Two-SM variant for plain GEMMs (one tap, one phase, K a multiple of 64):
// a cluster of two CTAs computes 256 x 256 output tiles with
// tcgen05.mma.cta_group::2.  CTA r of the pair stages rows [128r, 128r+128)
// of the tile's A rows and of its B rows (its half of N): 32 KB per 64-deep
// K step, and every A and B byte a pair reads from L2 feeds 256 rows or
// columns instead of 128.  CTA r holds rows [128r, +128) of the fp32
// accumulator (two accumulators of 256 columns: all 512 TMEM columns).  The
// leader (rank 0) counts both CTAs' copy bytes on its barriers, issues the
// pair MMAs and commits to both CTAs' barriers; both CTAs run the epilogue
// of their rows and release an accumulator by arriving on the leader's
// barrier.
//
// Epilogue (tma_epi != 0): a lane holds one output row, so direct stores
// touch 32 rows (32 cache lines) per instruction.  Instead each warp writes
// its 32-row chunk into a 128-byte-row shared-memory tile in the 128-byte
// swizzle (16-byte unit j of row r at unit j ^ (r & 7): conflict-free) and
// one lane hands the tile to a TMA bulk store, which also clips the tile at
// M and N.  Two 4 KB tiles per warp alternate; a tile is rewritten only after
// the bulk store issued from it has read it.  An fp32 residual arrives the
// same way, one chunk ahead, into the tile the result then overwrites.
constexpr int kPairBN = 256;
constexpr int kPairBK = 64;
constexpr int kPairStages = 4;
constexpr uint32_t kStageTile = 4096;  // 32 rows x 128 bytes

// Bias of 16 output columns starting at n0 (0 past N or without bias).
__device__ __forceinline__ void bias16(const TcEpilogue& e, int n0, int N, bool vec, float* bb) {
  if (e.bias && vec && n0 + 16 <= N) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(e.bias + n0 + j));
      bb[j] = v.x;
      bb[j + 1] = v.y;
      bb[j + 2] = v.z;
      bb[j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) bb[j] = (e.bias && n0 + j < N) ? __ldg(e.bias + n0 + j) : 0.f;
  }
}

// Address of 16-byte unit j of row r in a 1024-byte-aligned swizzled tile.
__device__ __forceinline__ uint8_t* swz_unit(uint8_t* tile, int r, int j) {
  return tile + r * 128 + ((j ^ (r & 7)) << 4);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                     const TcProblem prob, const TcEpilogue epi, uint32_t* status) {
  const TcProblem p = prob;
  const TcEpilogue e = epi;
  constexpr uint32_t kHalfBytes = 128u * kPairBK * 2u;  // 128 rows of A or of B, 16 KB
  constexpr uint32_t sbo = 8u * 128u;                    // 8-row atom stride (128 B rows)
  constexpr uint32_t idesc = idesc_f16_f32(256, kPairBN);
  constexpr int kAcc = 2;
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kPairStages * kHalfBytes;
  uint8_t* sOut = sB + kPairStages * kHalfBytes;  // kEpiWarps x 2 staging tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + kEpiWarps * 2 * kStageTile);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;
  uint64_t* tempty = tfull + kAcc;
  uint64_t* rbar = tempty + kAcc;  // kEpiWarps x 2: residual tile landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + kEpiWarps * 2);

  const uint32_t rank = cluster_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (p.M + 255) / 256, n_tiles = (p.N + kPairBN - 1) / kPairBN;
  const int tiles = m_tiles * n_tiles;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int kbn = p.kc / kPairBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);  // the epilogue warps of both CTAs
    }
    for (int w = 0; w < 2 * kEpiWarps; ++w) mbar_init(&rbar[w], 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.tma_epi) prefetch_tmap(&tmC);
    if (p.tma_epi == 2 && e.residual) prefetch_tmap(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers and TMEM exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Programmatic dependent launch: the set-up above and (B being weights no
  // kernel in the stream writes) the first stages' B loads overlap the
  // previous kernel; activations, bias, residual and outputs are touched only
  // after griddep_wait (a no-op for an ordinary launch).
  const int pre = (p.pdl && pair < tiles) ? (kbn < kPairStages ? kbn : kPairStages) : 0;
  if (warp == 0 && lane == 0 && pre > 0) {
    const int nt0 = pair % n_tiles;
    for (int s = 0; s < pre; ++s) {
      if (rank == 0) mbar_arrive_expect_tx(&full[s], 4u * kHalfBytes);  // both CTAs' A and B
      tma_load_2d_pair(sB + static_cast<size_t>(s) * kHalfBytes, &tmB, cluster_addr(&full[s], 0),
                       s * kPairBK, nt0 * kPairBN + static_cast<int>(rank) * 128);
    }
  }
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        const int mt = tile / n_tiles, nt = tile - (tile / n_tiles) * n_tiles;
        for (int kb = 0; kb < kbn; ++kb, ++it) {
          const int s = it % kPairStages;
          const uint32_t ph = static_cast<uint32_t>(it / kPairStages) & 1u;
          const uint32_t lead_full = cluster_addr(&full[s], 0);
          if (it < pre) {  // B and the expected bytes went out before griddep_wait
            tma_load_2d_pair(sA + static_cast<size_t>(s) * kHalfBytes, &tmA, lead_full,
                             kb * kPairBK, mt * 256 + static_cast<int>(rank) * 128);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1u, status)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 4u * kHalfBytes);  // both CTAs' A and B
          tma_load_2d_pair(sA + static_cast<size_t>(s) * kHalfBytes, &tmA, lead_full, kb * kPairBK,
                           mt * 256 + static_cast<int>(rank) * 128);
          tma_load_2d_pair(sB + static_cast<size_t>(s) * kHalfBytes, &tmB, lead_full, kb * kPairBK,
                           nt * kPairBN + static_cast<int>(rank) * 128);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------- MMA issuer (leader only)
      int it = 0, tl = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs, ++tl) {
        const int acc = tl & 1;
        const uint32_t aph = static_cast<uint32_t>(tl >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * kPairBN);
        for (int kb = 0; kb < kbn; ++kb, ++it) {
          const int s = it % kPairStages;
          const uint32_t ph = static_cast<uint32_t>(it / kPairStages) & 1u;
          if (!mbar_wait(&full[s], ph, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + static_cast<size_t>(s) * kHalfBytes);
          const uint32_t b_base = smem_u32(sB + static_cast<size_t>(s) * kHalfBytes);
#pragma unroll
          for (int j = 0; j < kPairBK / 16; ++j)
            tc_mma_f16_pair(d_tmem, smem_desc(a_base + 32u * j, sbo, 2),
                            smem_desc(b_base + 32u * j, sbo, 2), idesc, (kb | j) ? 1u : 0u);
          tc_commit_pair(cluster_addr(&empty[s], 0));  // both CTAs may refill stage s
          tc_commit_pair(cluster_addr(&empty[s], 1));
        }
        if (!ok) break;
        tc_commit_pair(cluster_addr(&tfull[acc], 0));  // both CTAs' rows of the tile are done
        tc_commit_pair(cluster_addr(&tfull[acc], 1));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;      // TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;  // column half
    const int cbeg = half * (kPairBN / 2);
    const bool bias_vec = e.bias && aligned16(e.bias);
    uint8_t* stile = sOut + static_cast<size_t>(warp - 2) * 2 * kStageTile;
    uint64_t* rb = rbar + (warp - 2) * 2;
    const bool res_tma = p.tma_epi == 2 && e.residual != nullptr;
    int cc = 0;        // staging tiles used so far (tile cc & 1 next)
    uint32_t rph = 0;  // residual barrier parities
    int tl = 0;
    for (int tile = pair; tile < tiles; tile += npairs, ++tl) {
      const int mt = tile / n_tiles, nt = tile - (tile / n_tiles) * n_tiles;
      const int acc = tl & 1;
      const uint32_t aph = static_cast<uint32_t>(tl >> 1) & 1u;
      const int row0 = mt * 256 + static_cast<int>(rank) * 128 + quarter * 32;
      const int i = row0 + lane;
      const bool row_ok = i < p.M;
      const long long orow = i;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * kPairBN);
      if (p.tma_epi == 0) {
        float bnext[16], rnext[16], snext[16];
        fetch16(e, row_ok, orow, nt * kPairBN + cbeg, p.N, 0, bias_vec, bnext, rnext, snext);
        if (!mbar_wait(&tfull[acc], aph, status)) break;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + kPairBN / 2; c0 += 16) {
          float bcur[16], rcur[16], scur[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            bcur[j] = bnext[j];
            rcur[j] = rnext[j];
            scur[j] = snext[j];
          }
          if (c0 + 16 < cbeg + kPairBN / 2)
            fetch16(e, row_ok, orow, nt * kPairBN + c0 + 16, p.N, 0, bias_vec, bnext, rnext, snext);
          uint32_t r[16];
          tmem_ld16(t_row + static_cast<uint32_t>(c0), r);
          tmem_ld_wait();
          if (row_ok && nt * kPairBN + c0 < p.N)
            store16(e, orow, nt * kPairBN + c0, p.N, r, 0, bcur, rcur, scur);
        }
      } else if (p.tma_epi == 1) {
        // fp16 output, 64-column chunks
        if (!mbar_wait(&tfull[acc], aph, status)) break;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + kPairBN / 2; c0 += 64) {
          const int n0 = nt * kPairBN + c0;
          if (n0 >= p.N) break;
          if (e.vt && n0 + 64 > e.vt_c0) {  // V^T columns: scattered per-head stores
#pragma unroll 1
            for (int q = 0; q < 4; ++q) {
              float bb[16], rr[16], ss[16];
              fetch16(e, row_ok, orow, n0 + 16 * q, p.N, 0, bias_vec, bb, rr, ss);
              uint32_t r[16];
              tmem_ld16(t_row + static_cast<uint32_t>(c0 + 16 * q), r);
              tmem_ld_wait();
              if (row_ok && n0 + 16 * q < p.N) store16(e, orow, n0 + 16 * q, p.N, r, 0, bb, rr, ss);
            }
            continue;
          }
          uint8_t* st = stile + (cc & 1) * kStageTile;
          if (lane == 0) bulk_wait_read<1>();  // the store issued from `st` has read it
          __syncwarp();
#pragma unroll 1
          for (int q = 0; q < 4; ++q) {
            uint32_t r[16];
            float v[16], bb[16];
            tmem_ld16(t_row + static_cast<uint32_t>(c0 + 16 * q), r);
            bias16(e, n0 + 16 * q, p.N, bias_vec, bb);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = fmaf(__uint_as_float(r[j]), e.alpha, bb[j]);
            act_array<16>(v, e.act, e.slope);
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) pk[j] = f2h2(v[2 * j], v[2 * j + 1]);
            *reinterpret_cast<uint4*>(swz_unit(st, lane, 2 * q)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(swz_unit(st, lane, 2 * q + 1)) =
                make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, st, n0, row0);
            bulk_commit();
          }
          ++cc;
        }
      } else {
        // fp32 output (+ fp32 residual), 32-column chunks
        const int nfirst = nt * kPairBN + cbeg;
        if (res_tma && lane == 0 && nfirst < p.N) {
          bulk_wait_read<1>();  // the store issued from tile cc & 1 has read it
          mbar_arrive_expect_tx(&rb[cc & 1], kStageTile);
          tma_load_2d(stile + (cc & 1) * kStageTile, &tmR, &rb[cc & 1], nfirst, row0);
        }
        if (!mbar_wait(&tfull[acc], aph, status)) break;
        tc_fence_after();
        bool ok = true;
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + kPairBN / 2 && ok; c0 += 32) {
          const int n0 = nt * kPairBN + c0;
          if (n0 >= p.N) break;
          const int b = cc & 1;
          uint8_t* st = stile + b * kStageTile;
          if (res_tma) {
            if (lane == 0 && c0 + 32 < cbeg + kPairBN / 2 && n0 + 32 < p.N) {
              bulk_wait_read<0>();  // the previous chunk's store has read tile b ^ 1
              mbar_arrive_expect_tx(&rb[b ^ 1], kStageTile);
              tma_load_2d(stile + (b ^ 1) * kStageTile, &tmR, &rb[b ^ 1], n0 + 32, row0);
            }
            const uint32_t par = (rph >> b) & 1u;
            bool got = true;
            if (lane == 0) got = mbar_wait(&rb[b], par, status);
            got = __shfl_sync(0xffffffffu, got, 0) != 0;
            if (!got) {
              ok = false;
              break;
            }
            mbar_wait(&rb[b], par, status);  // complete: each lane's own acquire of the tile
            rph ^= 1u << b;
          } else {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
          }
#pragma unroll 1
          for (int q = 0; q < 2; ++q) {
            uint32_t r[16];
            float v[16], bb[16];
            tmem_ld16(t_row + static_cast<uint32_t>(c0 + 16 * q), r);
            bias16(e, n0 + 16 * q, p.N, bias_vec, bb);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = fmaf(__uint_as_float(r[j]), e.alpha, bb[j]);
            act_array<16>(v, e.act, e.slope);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float4* u = reinterpret_cast<float4*>(swz_unit(st, lane, 4 * q + k));
              float4 o = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
              if (res_tma) {
                const float4 rv = *u;
                o.x = fmaf(e.res_scale, rv.x, o.x);
                o.y = fmaf(e.res_scale, rv.y, o.y);
                o.z = fmaf(e.res_scale, rv.z, o.z);
                o.w = fmaf(e.res_scale, rv.w, o.w);
              }
              *u = o;
            }
          }
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, st, n0, row0);
            bulk_commit();
          }
          ++cc;
        }
        if (!ok) break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));
    }
    if (lane == 0) bulk_wait<0>();  // every bulk store of this warp written
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's last MMAs wrote this CTA's TMEM and read its tiles
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

size_t pair_smem_bytes() {
  return 1024 + static_cast<size_t>(kPairStages) * 2 * 128 * kPairBK * 2 +
         static_cast<size_t>(kEpiWarps) * 2 * kStageTile +
         (2 * kPairStages + 4 + 2 * kEpiWarps) * 8 + 16;
}

int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                const CUtensorMap& tr, const TcProblem& p, const TcEpilogue& e, cudaStream_t st) {
  const size_t smem = pair_smem_bytes();
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(gemm_pair_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem)),
                        "cudaFuncSetAttribute(gemm_pair)");
    if (rc) return rc;
    attr_set[dev] = true;
  }
  const long long tiles = static_cast<long long>((p.M + 255) / 256) * ((p.N + kPairBN - 1) / kPairBN);
  const int pairs = static_cast<int>(std::min<long long>(tiles, sm_count() / 2));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = p.pdl ? 2 : 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, gemm_pair_kernel, ta, tb, tc, tr, p, e, device_status()),
                    "gemm_pair_kernel launch");
}

template <int BN>
int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to32,
              const CUtensorMap& to16, const CUtensorMap& to16a, const CUtensorMap& tmean,
              const TcProblem& p, const TcEpilogue& e, cudaStream_t st) {
  int stages;
  size_t smem;
  // the bulk-copy epilogue's buffers come out of the stage budget
  const size_t budget = kSmemBudget - (p.bulk_epi ? kBulkStgBytes + 1024 : 0);
  if (p.win) {  // window stages + every tap's weights (tc_run checked that two stages fit)
    const size_t a_win = (static_cast<size_t>(p.win) * p.bk * 2 + 1023) & ~static_cast<size_t>(1023);
    const size_t b_all = static_cast<size_t>(p.taps) * BN * p.bk * 2;
    stages = static_cast<int>(std::min<size_t>(8, (budget - b_all) / a_win));
    smem = 1024 + stages * a_win + b_all + (2 * stages + 9) * 8 + 16;
  } else {
    const int stage_bytes = (kBM + BN) * p.bk * 2;
    stages = std::max(2, std::min(static_cast<int>(budget) / stage_bytes, 8));
    smem = 1024 + static_cast<size_t>(stages) * stage_bytes + (2 * stages + 9) * 8 + 16;
  }
  if (p.bulk_epi) smem += 1024 + kBulkStgBytes;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(gemm_tc_kernel<BN>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBudget + 8192),
                        "cudaFuncSetAttribute(gemm_tc)");
    if (rc) return rc;
    attr_set[dev] = true;
  }
  const long long tiles = static_cast<long long>((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) *
                          p.phases;
  const int grid = static_cast<int>(std::min<long long>(tiles, sm_count()));
  if (p.pdl)
    return launch_pdl(gemm_tc_kernel<BN>, dim3(grid), dim3(kThreads), smem, st, "gemm_tc_kernel",
                      ta, tb, to32, to16, to16a, tmean, p, e, stages, device_status());
  gemm_tc_kernel<BN><<<grid, kThreads, smem, st>>>(ta, tb, to32, to16, to16a, tmean, p, e, stages,
                                                   device_status());
  return check_launch("gemm_tc_kernel");
}

// CUDA-core path for shapes the TMA descriptors cannot express: one thread
// per (row, 16-column group), fp32 FMA over K, the same epilogue.
__global__ void gemm_simt_kernel(const uint16_t* __restrict__ a, long long lda,
                                 const uint16_t* __restrict__ b, long long ldb, int M, int N, int K,
                                 const TcEpilogue epi) {
  const TcEpilogue e = epi;  // register copy (stores below must not re-read parameter space)
  const int groups = (N + 15) / 16;
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long long>(M) * groups) return;
  const int m = static_cast<int>(idx / groups), g = static_cast<int>(idx % groups);
  uint32_t r[16];
  const uint16_t* ar = a + m * lda;
  for (int j = 0; j < 16; ++j) {
    const int n = g * 16 + j;
    float acc = 0.f;
    if (n < N) {
      const uint16_t* br = b + n * ldb;
      for (int k = 0; k < K; ++k) acc = fmaf(h2f(ar[k]), h2f(br[k]), acc);
    }
    r[j] = __float_as_uint(acc);
  }
  float bb[16], rr[16], ss[16];
  fetch16(e, true, m, g * 16, N, 0, false, bb, rr, ss);
  store16(e, m, g * 16, N, r, 0, bb, rr, ss);
}

int pick_bk(long long kc) {
  if (kc <= 16) return 16;
  if (kc <= 32) return 32;
  return 64;
}

CUtensorMapSwizzle swizzle_for(int bk) {
  return bk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                  : (bk == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

}  // namespace

int make_kmajor_map(CUtensorMap* map, const uint16_t* base, long long rows, long long kc,
                    long long ld, int box_rows, int bk) {
  const uint64_t dims[2] = {static_cast<uint64_t>(kc), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 2};
  const uint32_t box[2] = {static_cast<uint32_t>(bk), static_cast<uint32_t>(box_rows)};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(base), dims,
                      strides, box, swizzle_for(bk));
}

int tc_pick_bn(long long M, long long N) {
  if (N <= 16) return 16;
  if (N <= 32) return 32;
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  const long long m_tiles = (M + kBM - 1) / kBM;
  // 256-wide tiles halve A re-reads; keep them only while they still fill the GPU.
  return (m_tiles * ((N + 255) / 256) >= sm_count()) ? 256 : 128;
}

// One-SM kernel's bulk-copy epilogue where the outputs allow it
// (gsvk_gemm_set_bulk_epilogue).
static int g_bulk_epi = 1;
// Two-SM GEMM for eligible plain problems (gsvk_gemm_set_pair): 0 never,
// 1 when pair_wins, 2 always.
static int g_pair_mode = 1;

// Whether the two-SM kernel beats the one-SM kernel with BN-wide tiles.  Both
// are bound by each SM's L2 ingest (~64 B/clk) rather than by the tensor pipe:
// per 64-deep K block a pair SM loads 32 KB for a 128x256 slice (512 clk), a
// one-SM CTA 48 KB at BN = 256 (768 clk) or 32 KB at BN = 128 (512 clk for
// half the work).  Cost = tile rounds x K-block cost; on a tie the pair wins
// only for long K, where its larger unoverlapped epilogue is amortised.
static bool pair_wins(long long M, long long N, long long K, int bn) {
  const long long sms = sm_count(), pairs = sms / 2;
  const long long t2 = ((M + 255) / 256) * ((N + 255) / 256);
  const long long t1 = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  const long long pair_cost = ((t2 + pairs - 1) / pairs) * 512;
  const long long one_cost = ((t1 + sms - 1) / sms) * (bn >= 256 ? 768 : 512);
  return pair_cost < one_cost || (pair_cost == one_cost && K >= 2048);
}

int tc_run(const uint16_t* a, long long a_rows, long long lda, const uint16_t* b,
           long long b_rows, long long ldb, TcProblem p, const TcEpilogue& e, int bn,
           cudaStream_t st, long long a_cols, long long b_cols) {
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  if (p.kc % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0)
    return fail(GSVK_ERR_ALIGN, "tensor-core path needs K and leading dims multiple of 8");
  if (!aligned16(a) || !aligned16(b))
    return fail(GSVK_ERR_ALIGN, "tensor-core path needs 16-byte aligned A and B");
  if (p.M <= 0 || p.N <= 0 || p.kc <= 0 || p.taps <= 0)
    return fail(GSVK_ERR_INVALID, "empty GEMM");
  p.bk = pick_bk(p.kc);
  const bool bn_auto = bn == 0;
  if (bn == 0) bn = tc_pick_bn(p.M, p.N);
  // window mode: a dilated conv with one K block per tap and one column tile,
  // whose input window (<= 256 rows, the TMA box limit) and weights fit
  p.win = 0;
  if (!p.convt && p.bh == 0 && p.phases == 1 && p.taps > 1 && p.kc <= p.bk && bn >= p.N) {
    const long long R = kBM + static_cast<long long>(p.taps - 1) * p.dil;
    const long long a_win = (R * p.bk * 2 + 1023) & ~1023LL;
    const long long b_all = static_cast<long long>(p.taps) * bn * p.bk * 2;
    if (R <= 256 && b_all + 2 * a_win <= kSmemBudget) p.win = static_cast<int>(R);
  }
  CUtensorMap ta, tb;
  if (g_pair_mode && (bn_auto || bn == 256) && !p.convt && p.bh == 0 && p.phases == 1 &&
      p.taps == 1 && p.win == 0 && p.kc % kPairBK == 0 && p.M >= 256 && p.N >= 256 &&
      a_cols == 0 && b_cols == 0 && (g_pair_mode == 2 || pair_wins(p.M, p.N, p.kc, bn))) {
    p.bk = kPairBK;
    int rc = make_kmajor_map(&ta, a, a_rows, p.kc, lda, 128, kPairBK);
    if (!rc) rc = make_kmajor_map(&tb, b, b_rows, p.kc, ldb, 128, kPairBK);
    if (rc) return rc;
    // bulk-copy epilogue for a single fp16 or fp32 output (32-row tiles of
    // 128-byte rows: 64 fp16 or 32 fp32 columns)
    CUtensorMap tc{}, tr{};
    p.tma_epi = 0;
    const uint64_t odims[2] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M)};
    if (e.c16 && !e.c32 && !e.c16_act && !e.mean_sum && !e.residual && aligned16(e.c16) &&
        e.ld_c16 % 8 == 0) {
      const uint64_t str[1] = {static_cast<uint64_t>(e.ld_c16) * 2};
      const uint32_t box[2] = {64, 32};
      rc = encode_tiled(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, e.c16, odims, str, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      p.tma_epi = 1;
    } else if (e.c32 && !e.c16 && !e.c16_act && !e.mean_sum && !e.vt && aligned16(e.c32) &&
               e.ld_c32 % 4 == 0 &&
               (!e.residual || (aligned16(e.residual) && e.ld_res % 4 == 0))) {
      const uint32_t box[2] = {32, 32};
      const uint64_t str[1] = {static_cast<uint64_t>(e.ld_c32) * 4};
      rc = encode_tiled(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, e.c32, odims, str, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
      if (!rc && e.residual) {
        const uint64_t rstr[1] = {static_cast<uint64_t>(e.ld_res) * 4};
        rc = encode_tiled(&tr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(e.residual),
                          odims, rstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
      }
      if (rc) return rc;
      p.tma_epi = 2;
    }
    return launch_pair(ta, tb, tc, tr, p, e, st);
  }
  int rc = make_kmajor_map(&ta, a, a_rows, a_cols ? a_cols : p.kc, lda, p.win ? p.win : kBM, p.bk);
  if (rc) return rc;
  rc = make_kmajor_map(&tb, b, b_rows, b_cols ? b_cols : p.kc, ldb, bn, p.bk);
  if (rc) return rc;
  // bulk-copy epilogue: contiguous output rows (no ConvT interleave, no
  // batched offsets), no transposed-V output, 16-byte aligned outputs, and
  // the stage ring still two deep in the smaller budget
  CUtensorMap to32{}, to16{}, to16a{}, tmean{};
  p.bulk_epi = 0;
  if (g_bulk_epi && !p.convt && p.bh == 0 && p.phases == 1 && !e.vt &&
      (e.c32 || e.c16 || e.c16_act || e.mean_sum) &&
      (!e.c32 || (aligned16(e.c32) && e.ld_c32 % 4 == 0)) &&
      (!e.mean_sum || (aligned16(e.mean_sum) && e.ld_c32 % 4 == 0)) &&
      (!e.c16 || (aligned16(e.c16) && e.ld_c16 % 8 == 0)) &&
      (!e.c16_act || (aligned16(e.c16_act) && e.ld_c16_act % 8 == 0))) {
    const long long budget = kSmemBudget - static_cast<long long>(kBulkStgBytes) - 1024;
    long long need = 2LL * (kBM + bn) * p.bk * 2;
    if (p.win) {
      const long long a_win = (static_cast<long long>(p.win) * p.bk * 2 + 1023) & ~1023LL;
      need = static_cast<long long>(p.taps) * bn * p.bk * 2 + 2 * a_win;
    }
    if (need <= budget) {
      const uint64_t odims[2] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M)};
      const uint32_t box[2] = {16, 32};
      if (e.c32) {
        const uint64_t str[1] = {static_cast<uint64_t>(e.ld_c32) * 4};
        rc = encode_tiled(&to32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, e.c32, odims, str, box,
                          CU_TENSOR_MAP_SWIZZLE_64B);
      }
      if (!rc && e.c16) {
        const uint64_t str[1] = {static_cast<uint64_t>(e.ld_c16) * 2};
        rc = encode_tiled(&to16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, e.c16, odims, str, box,
                          CU_TENSOR_MAP_SWIZZLE_32B);
      }
      if (!rc && e.c16_act) {
        const uint64_t str[1] = {static_cast<uint64_t>(e.ld_c16_act) * 2};
        rc = encode_tiled(&to16a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, e.c16_act, odims, str, box,
                          CU_TENSOR_MAP_SWIZZLE_32B);
      }
      if (!rc && e.mean_sum) {  // the running mean shares the fp32 output's layout
        const uint64_t str[1] = {static_cast<uint64_t>(e.ld_c32) * 4};
        rc = encode_tiled(&tmean, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, e.mean_sum, odims, str, box,
                          CU_TENSOR_MAP_SWIZZLE_64B);
      }
      if (rc) return rc;
      p.bulk_epi = 1;
    }
  }
  switch (bn) {
    case 16: return launch_bn<16>(ta, tb, to32, to16, to16a, tmean, p, e, st);
    case 32: return launch_bn<32>(ta, tb, to32, to16, to16a, tmean, p, e, st);
    case 64: return launch_bn<64>(ta, tb, to32, to16, to16a, tmean, p, e, st);
    case 128: return launch_bn<128>(ta, tb, to32, to16, to16a, tmean, p, e, st);
    case 256: return launch_bn<256>(ta, tb, to32, to16, to16a, tmean, p, e, st);
    default: return fail(GSVK_ERR_INVALID, "bad BN %d", bn);
  }
}

int simt_gemm(const gsvk_gemm_args* g, const TcEpilogue& e, cudaStream_t st) {
  const long long groups = (static_cast<long long>(g->N) + 15) / 16;
  const long long threads = static_cast<long long>(g->M) * groups;
  gemm_simt_kernel<<<static_cast<unsigned>((threads + 127) / 128), 128, 0, st>>>(
      g->a, (long long)g->lda, g->b, (long long)g->ldb, (int)g->M, (int)g->N, (int)g->K, e);
  return check_launch("gemm_simt_kernel");
}

TcEpilogue make_epilogue() {
  TcEpilogue e{};
  e.alpha = 1.f;
  e.res_scale = 1.f;
  return e;
}

}  // namespace gsvk

using namespace gsvk;

extern "C" {

int gsvk_gemm_f16(const uint16_t* a, const uint16_t* b, float* c, size_t M, size_t N, size_t K,
                  gsvk_stream_t stream) {
  gsvk_gemm_args g{};
  g.a = a;
  g.lda = K;
  g.b = b;
  g.ldb = K;
  g.M = M;
  g.N = N;
  g.K = K;
  g.c = c;
  g.ldc = N;
  g.alpha = 1.f;
  return gsvk_gemm_f16_ex(&g, stream);
}

int gsvk_gemm_f16_ex(const gsvk_gemm_args* g, gsvk_stream_t stream) {
  return gemm_ex_run(g, as_cuda(stream), false);
}

int gsvk_gemm_uses_pair(size_t M, size_t N, size_t K) {
  if (M == 0 || N == 0 || K == 0 || M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff || K % 8)
    return 0;
  const void* aligned = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  if (gsvk::skinny_fits((long long)M, (long long)N, (long long)K, (long long)K, (long long)K,
                        aligned, aligned))
    return 0;  // few rows: the split-K kernel
  if (!g_pair_mode || K % gsvk::kPairBK != 0 || M < 256 || N < 256) return 0;
  return (g_pair_mode == 2 ||
          gsvk::pair_wins((long long)M, (long long)N, (long long)K,
                          gsvk::tc_pick_bn((long long)M, (long long)N)))
             ? 1
             : 0;
}

int gsvk_gemm_set_bulk_epilogue(int enable) {
  g_bulk_epi = enable != 0;
  return GSVK_OK;
}

int gsvk_gemm_set_pair(int mode) {
  if (mode < 0 || mode > 2) return gsvk::fail(GSVK_ERR_INVALID, "gemm_set_pair: mode %d", mode);
  g_pair_mode = mode;
  return GSVK_OK;
}

int gsvk_gemm_f16_batched(const gsvk_gemm_args* g, size_t batch, size_t stride_a,
                          size_t stride_b, size_t stride_c, gsvk_stream_t stream) {
  if (!g || batch == 0) return fail(GSVK_ERR_INVALID, "gemm_batched: null arguments or zero batch");
  if (!g->a || !g->b || (!g->c && !g->c_f16) || g->M == 0 || g->N == 0 || g->K == 0)
    return fail(GSVK_ERR_INVALID, "gemm_batched: null pointer or zero size");
  cudaStream_t st = as_cuda(stream);
  const size_t lda = g->lda ? g->lda : g->K, ldb = g->ldb ? g->ldb : g->K;
  const size_t ldc = g->ldc ? g->ldc : g->N, ldh = g->ldc_f16 ? g->ldc_f16 : g->N;
  const size_t ldr = g->ld_res ? g->ld_res : g->N;
  if (lda < g->K || ldb < g->K) return fail(GSVK_ERR_INVALID, "gemm_batched: lda/ldb < K");
  if (g->act < GSVK_ACT_NONE || g->act > GSVK_ACT_TANH)
    return fail(GSVK_ERR_INVALID, "gemm_batched: bad act");
  // One persistent tensor-core launch over every (problem, tile) when the
  // problems sit at whole-row strides of one tensor each and every output
  // shares one row layout; otherwise one launch per problem.
  const size_t ldo = g->c ? ldc : ldh;
  bool one_launch = g->K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0 && aligned16(g->a) &&
                    aligned16(g->b) && stride_a % lda == 0 && stride_b % ldb == 0 &&
                    stride_c % ldo == 0 && (!g->c || !g->c_f16 || ldc == ldh) &&
                    (!g->residual || ldr == ldo);
  const size_t a_rb = one_launch ? stride_a / lda : 0, b_rb = one_launch ? stride_b / ldb : 0,
               c_rb = one_launch ? stride_c / ldo : 0;
  one_launch = one_launch && (batch - 1) * a_rb + g->M < 0x7fffffffULL &&
               (batch - 1) * b_rb + g->N < 0x7fffffffULL &&
               (batch - 1) * c_rb + g->M < 0x7fffffffULL && batch < 0x7fffffffULL &&
               c_rb >= g->M;  // outputs of different problems must not overlap
  if (!one_launch) {
    for (size_t i = 0; i < batch; ++i) {
      gsvk_gemm_args gi = *g;
      gi.a += i * stride_a;
      gi.b += i * stride_b;
      if (gi.c) gi.c += i * stride_c;
      if (gi.c_f16) gi.c_f16 += i * stride_c;
      if (gi.residual) gi.residual += i * stride_c;
      if (int rc = gemm_ex_run(&gi, st, false)) return rc;
    }
    return GSVK_OK;
  }
  TcEpilogue e = make_epilogue();
  e.bias = g->bias;
  e.residual = g->residual;
  e.ld_res = (long long)ldr;
  e.c32 = g->c;
  e.ld_c32 = (long long)ldc;
  e.c16 = g->c_f16;
  e.ld_c16 = (long long)ldh;
  e.act = g->act;
  e.slope = g->slope;
  e.alpha = g->alpha == 0.f ? 1.f : g->alpha;
  TcProblem p{};
  p.M = (int)g->M;
  p.N = (int)g->N;
  p.kc = (int)g->K;
  p.taps = 1;
  p.dil = 1;
  p.phases = (int)batch;
  p.out_rows = (int)g->M;
  p.bh = 1;  // phase = problem index
  p.a_rb = (int)a_rb;
  p.b_rb = (int)b_rb;
  p.c_rb = (int)c_rb;
  const long long m_tiles = (long long)((g->M + 127) / 128);
  const int bn = g->N <= 128 ? 0 : (m_tiles * (long long)((g->N + 255) / 256) * (long long)batch >=
                                            sm_count() ? 256 : 128);
  return tc_run(g->a, (long long)((batch - 1) * a_rb + g->M), (long long)lda, g->b,
                (long long)((batch - 1) * b_rb + g->N), (long long)ldb, p, e, bn, st);
}

}  // extern "C"

int gsvk::gemm_ex_run(const gsvk_gemm_args* args, cudaStream_t st, bool static_b) {
  if (!args) return fail(GSVK_ERR_INVALID, "gemm: null arguments");
  gsvk_gemm_args norm = *args;  // zero leading dimensions mean dense rows
  if (!norm.lda) norm.lda = norm.K;
  if (!norm.ldb) norm.ldb = norm.K;
  const gsvk_gemm_args* g = &norm;
  if (!g->a || !g->b || (!g->c && !g->c_f16) || g->M == 0 || g->N == 0 || g->K == 0)
    return fail(GSVK_ERR_INVALID, "gemm: null pointer or zero size");
  if (g->M > 0x7fffffff || g->N > 0x7fffffff || g->K > 0x7fffffff)
    return fail(GSVK_ERR_UNSUPPORTED, "gemm: size > 2^31");
  if (g->lda < g->K || g->ldb < g->K) return fail(GSVK_ERR_INVALID, "gemm: lda/ldb < K");
  if (g->act < GSVK_ACT_NONE || g->act > GSVK_ACT_TANH) return fail(GSVK_ERR_INVALID, "bad act");
  TcEpilogue e = make_epilogue();
  e.bias = g->bias;
  e.residual = g->residual;
  e.ld_res = g->ld_res ? (long long)g->ld_res : (long long)g->N;
  e.c32 = g->c;
  e.ld_c32 = g->ldc ? (long long)g->ldc : (long long)g->N;
  e.c16 = g->c_f16;
  e.ld_c16 = g->ldc_f16 ? (long long)g->ldc_f16 : (long long)g->N;
  e.act = g->act;
  e.slope = g->slope;
  e.alpha = g->alpha == 0.f ? 1.f : g->alpha;
  if (g->K % 8 != 0 || g->lda % 8 != 0 || g->ldb % 8 != 0 || !aligned16(g->a) ||
      !aligned16(g->b))
    return simt_gemm(g, e, st);  // odd K (conv K=7/9, test shapes)
  // few rows (decode steps, the FFN-up of one 128-token chunk): split-K cluster kernel
  if (skinny_fits((long long)g->M, (long long)g->N, (long long)g->K, (long long)g->lda,
                  (long long)g->ldb, g->a, g->b))
    return skinny_run(g->a, (int)g->M, (long long)g->lda, g->b, (int)g->N, (long long)g->ldb,
                      (int)g->K, e, st, static_b);
  TcProblem p{};
  p.M = (int)g->M;
  p.N = (int)g->N;
  p.kc = (int)g->K;
  p.taps = 1;
  p.dil = 1;
  p.pad = 0;
  p.b_tap_rows = 0;
  p.convt = 0;
  p.phases = 1;
  p.out_rows = (int)g->M;
  p.pdl = static_b ? 1 : 0;
  return tc_run(g->a, (long long)g->M, (long long)g->lda, g->b, (long long)g->N,
                (long long)g->ldb, p, e, 0, st);
}
