// gemm_skinny.cu — tensor-core GEMM for few-row activations (decode steps:
// M = batch <= 128), C[m, n] = epi( sum_k X[m, k] * W[n, k] ).
//
// With M this small the job is streaming W from HBM, so the problem is
// turned around ("swap AB"): each 128-row tile of W is the MMA's A operand
// (M = 128) and the activation rows are its N (Mp = M rounded up to 16), so
// no tensor-core row is spent on padding.  K is split across the CTAs of a
// thread-block cluster (up to 8): every CTA loads its K slice of the W tile
// and of X with TMA, accumulates in TMEM, and then owns 128/S rows of the
// tile: it reduces those rows over the S partials and applies the epilogue
// (bias, activation, residual, fp32/fp16 stores).
//
// The reduction is push-style: each CTA lays its partial out per destination
// rank and one thread bulk-copies every slice into the owner's receive
// buffer (completing the owner's mbarrier), so the reduce itself reads only
// local shared memory.  A split of 1 (whole K in one CTA) stores straight
// from TMEM.
//
// Launched with programmatic dependent launch: the W loads (constant data)
// are issued before griddepcontrol.wait, so they overlap the tail of the
// kernel that produces X.
#include <algorithm>

#include "gemm_tc.cuh"
#include "gsvk_internal.hpp"

namespace gsvk {

namespace {

constexpr int kSkThreads = 128;
constexpr int kSkBK = 64;             // K elements per stage (128-byte swizzle rows)
constexpr int kSkTileN = 128;         // W rows per tile (MMA M)
constexpr int kSkMaxSplit = 8;        // portable cluster size
constexpr int kSkMaxM = 128;          // activation rows (MMA N <= 128)
constexpr int kSkSmemBudget = 200 * 1024;
constexpr int kSkPre = 2;             // output groups per thread with prefetched operands

struct SkProblem {
  int M, N, K, Mp;
  int split;     // CTAs per cluster (K slices)
  int kb_total;  // K blocks of kSkBK
  int stages;    // K blocks per CTA (max)
  int v_bias, v_res, v_c32, v_c16, v_c16a;  // 16-byte (8 for fp16) vector access allowed
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Bulk copy from this CTA's shared memory to a cluster peer's, completing
// `bytes` transactions on the peer's mbarrier (both peer addresses from mapa).
__device__ __forceinline__ void bulk_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                             uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

// Epilogue of four adjacent outputs (m, n0..n0+3): y = act(alpha*acc + bias)
// + res_scale*residual, stored fp32 / fp16 / fp16(act2(y)), 16- or 8-byte
// accesses where the host allowed them.
struct SkOps {
  float4 bias, res;
};
__device__ __forceinline__ SkOps sk_ops(const SkProblem& p, const TcEpilogue& e, int m, int n0) {
  SkOps o{make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  const bool full = n0 + 3 < p.N;
  if (e.bias) {
    if (full && p.v_bias) {
      o.bias = __ldg(reinterpret_cast<const float4*>(e.bias + n0));
    } else {
      float* b = &o.bias.x;
      for (int u = 0; u < 4; ++u)
        if (n0 + u < p.N) b[u] = __ldg(e.bias + n0 + u);
    }
  }
  if (e.residual) {
    const float* rr = e.residual + m * e.ld_res + n0;
    if (full && p.v_res) {
      o.res = *reinterpret_cast<const float4*>(rr);
    } else {
      float* r = &o.res.x;
      for (int u = 0; u < 4; ++u)
        if (n0 + u < p.N) r[u] = rr[u];
    }
  }
  return o;
}
__device__ __forceinline__ void sk_store4(const SkProblem& p, const TcEpilogue& e, int m, int n0,
                                          float4 acc, const SkOps& o) {
  float v[4] = {fmaf(acc.x, e.alpha, o.bias.x), fmaf(acc.y, e.alpha, o.bias.y),
                fmaf(acc.z, e.alpha, o.bias.z), fmaf(acc.w, e.alpha, o.bias.w)};
  act_array<4>(v, e.act, e.slope);
  if (e.residual) {
    v[0] = fmaf(e.res_scale, o.res.x, v[0]);
    v[1] = fmaf(e.res_scale, o.res.y, v[1]);
    v[2] = fmaf(e.res_scale, o.res.z, v[2]);
    v[3] = fmaf(e.res_scale, o.res.w, v[3]);
  }
  const bool full = n0 + 3 < p.N;
  if (e.c32) {
    float* d = e.c32 + m * e.ld_c32 + n0;
    if (full && p.v_c32) {
      *reinterpret_cast<float4*>(d) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      for (int u = 0; u < 4; ++u)
        if (n0 + u < p.N) d[u] = v[u];
    }
  }
  if (e.c16) {
    uint16_t* d = e.c16 + m * e.ld_c16 + n0;
    if (full && p.v_c16) {
      *reinterpret_cast<uint2*>(d) = make_uint2(f2h2(v[0], v[1]),
                                                f2h2(v[2], v[3]));
    } else {
      for (int u = 0; u < 4; ++u)
        if (n0 + u < p.N) d[u] = f2h(v[u]);
    }
  }
  if (e.c16_act) {
    act_array<4>(v, e.act2, e.slope2);
    uint16_t* d = e.c16_act + m * e.ld_c16_act + n0;
    if (full && p.v_c16a) {
      *reinterpret_cast<uint2*>(d) = make_uint2(f2h2(v[0], v[1]),
                                                f2h2(v[2], v[3]));
    } else {
      for (int u = 0; u < 4; ++u)
        if (n0 + u < p.N) d[u] = f2h(v[u]);
    }
  }
}

// Split-1 epilogue: output column n, rows m0 .. m0+15 (one TMEM chunk).
__device__ __forceinline__ void sk_store_col16(const SkProblem& p, const TcEpilogue& e, int m0,
                                               int n, const uint32_t* r, float bias) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = fmaf(__uint_as_float(r[j]), e.alpha, bias);
  act_array<16>(v, e.act, e.slope);
  const int nm = min(16, p.M - m0);
  if (e.residual) {
    const float* rr = e.residual + static_cast<long long>(m0) * e.ld_res + n;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nm) v[j] = fmaf(e.res_scale, rr[j * e.ld_res], v[j]);
  }
  if (e.c32) {
    float* d = e.c32 + static_cast<long long>(m0) * e.ld_c32 + n;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nm) d[j * e.ld_c32] = v[j];
  }
  if (e.c16) {
    uint16_t* d = e.c16 + static_cast<long long>(m0) * e.ld_c16 + n;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nm) d[j * e.ld_c16] = f2h(v[j]);
  }
  if (e.c16_act) {
    act_array<16>(v, e.act2, e.slope2);
    uint16_t* d = e.c16_act + static_cast<long long>(m0) * e.ld_c16_act + n;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nm) d[j * e.ld_c16_act] = f2h(v[j]);
  }
}

// Shared memory (1 KB aligned): recv [split][Mp][rows_per] fp32 (filled by
// the cluster's bulk copies), then the TMA stages, whose space is reused as
// send [split][Mp][rows_per] once the MMAs have completed.
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       const SkProblem prob, const TcEpilogue epi, uint32_t* status) {
  // Register copies of the parameter structs: helpers take them by reference,
  // and a reference into parameter space would be re-read after every global
  // store (the compiler cannot rule out aliasing through the output pointers).
  const SkProblem p = prob;
  const TcEpilogue e = epi;
  extern __shared__ uint8_t sk_raw[];
  uint8_t* smem = align_smem<1024>(sk_raw);
  __shared__ uint64_t full[8], empty[8];
  __shared__ uint64_t done, recv_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int ok_flag;
  constexpr uint32_t w_bytes = kSkTileN * kSkBK * 2;  // 16 KB
  const uint32_t x_bytes = static_cast<uint32_t>(p.Mp) * kSkBK * 2;
  const uint32_t stage_bytes = w_bytes + x_bytes;
  const uint32_t tmem_cols = p.Mp <= 32 ? 32u : (p.Mp <= 64 ? 64u : 128u);
  const bool split = p.split > 1;
  const uint32_t tile_bytes = static_cast<uint32_t>(p.Mp) * kSkTileN * 4;  // one fp32 tile
  float* recv = reinterpret_cast<float*>(smem);
  uint8_t* stages = smem + (split ? tile_bytes : 0u);
  float* send = reinterpret_cast<float*>(stages);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = split ? cluster_ctarank() : 0u;
  const int tile = blockIdx.x / p.split;
  const int kb0 = static_cast<int>((static_cast<long long>(rank) * p.kb_total) / p.split);
  const int kb1 = static_cast<int>((static_cast<long long>(rank + 1) * p.kb_total) / p.split);
  const int nkb = kb1 - kb0;
  const int nst = min(nkb, p.stages);  // stage buffers (a ring when nkb > nst)
  const int rows_per = kSkTileN / p.split;  // >= 16
  const uint32_t slice_bytes = tile_bytes / static_cast<uint32_t>(p.split);

  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    mbar_init(&recv_bar, 1);
    fence_barrier_init();
    if (split) mbar_arrive_expect_tx(&recv_bar, tile_bytes);  // one slice from every rank
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (split) cluster_arrive();  // peers may target recv_bar once every rank has initialised it
  const uint32_t tmem = tmem_slot;

  bool ok = true;
  if (warp == 0) {
    // lane 0 streams the stages and issues the MMAs; lanes 1..31 park at the
    // warp barrier (spinning beside the issuing lane would slow it down)
    if (lane == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
    // W is constant: fetch it before the dependency on the producer of X resolves
    for (int s = 0; s < nst; ++s) {
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      tma_load_2d(stages + static_cast<size_t>(s) * stage_bytes, &tmW, &full[s], (kb0 + s) * kSkBK,
                  tile * kSkTileN);
    }
    griddep_wait();
    for (int s = 0; s < nst; ++s)
      tma_load_2d(stages + static_cast<size_t>(s) * stage_bytes + w_bytes, &tmX, &full[s],
                  (kb0 + s) * kSkBK, 0);
    const uint32_t idesc = idesc_f16_f32(kSkTileN, static_cast<uint32_t>(p.Mp));
    for (int i = 0; i < nkb && ok; ++i) {
      const int b = i % nst;
      const uint32_t ph = static_cast<uint32_t>(i / nst) & 1u;
      if (!mbar_wait(&full[b], ph, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a_base = smem_u32(stages + static_cast<size_t>(b) * stage_bytes);
      const uint32_t b_base = a_base + w_bytes;
#pragma unroll
      for (int j = 0; j < kSkBK / 16; ++j)
        tc_mma_f16(tmem, smem_desc(a_base + 32u * j, 1024, 2), smem_desc(b_base + 32u * j, 1024, 2),
                   idesc, (i | j) ? 1u : 0u);
      if (i + nst < nkb) {  // refill buffer b with K block i + nst once its MMAs have read it
        tc_commit(&empty[b]);
        if (!mbar_wait(&empty[b], ph, status)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[b], stage_bytes);
        uint8_t* dst = stages + static_cast<size_t>(b) * stage_bytes;
        tma_load_2d(dst, &tmW, &full[b], (kb0 + i + nst) * kSkBK, tile * kSkTileN);
        tma_load_2d(dst + w_bytes, &tmX, &full[b], (kb0 + i + nst) * kSkBK, 0);
      }
    }
    if (ok && nkb > 0) {
      tc_commit(&done);
      ok = mbar_wait(&done, 0, status);
    }
    ok_flag = ok ? 1 : 0;
    }
    __syncwarp();
  }
  griddep_wait();
  griddep_launch_dependents();

  const int nl = warp * 32 + lane;  // TMEM lane = W row of the tile
  if (!split) {
    // ------------------------------------------------ whole K in this CTA
    const int n = tile * kSkTileN + nl;
    const float bias = (e.bias && n < p.N) ? __ldg(e.bias + n) : 0.f;
    __syncthreads();  // thread 0 has seen the MMAs complete (the others wait here, idle)
    tc_fence_after();
    const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    for (int c0 = 0; c0 < p.Mp; c0 += 64) {  // up to four loads in flight per wait
      uint32_t r[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + 16 * u < p.Mp) tmem_ld16(t_row + static_cast<uint32_t>(c0 + 16 * u), r[u]);
      tmem_ld_wait();
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (n < p.N && c0 + 16 * u < p.M) sk_store_col16(p, e, c0 + 16 * u, n, r[u], bias);
    }
  } else {
    // ----------------------------------- split K: push slices, reduce own rows
    const int g4 = rows_per / 4;
    const int total = g4 * p.M;
    SkOps pre[kSkPre];
#pragma unroll
    for (int it = 0; it < kSkPre; ++it) {
      const int idx = tid + it * kSkThreads;
      const int m = idx / g4;
      const int n0 = tile * kSkTileN + static_cast<int>(rank) * rows_per + (idx % g4) * 4;
      pre[it] = (idx < total && n0 < p.N) ? sk_ops(p, e, m, n0)
                                           : SkOps{make_float4(0.f, 0.f, 0.f, 0.f),
                                                   make_float4(0.f, 0.f, 0.f, 0.f)};
    }
    // TMEM -> send[q][m][row] with q = nl / rows_per, row = nl % rows_per
    const int q = nl / rows_per, row = nl - (nl / rows_per) * rows_per;
    float* my = send + static_cast<size_t>(q) * p.Mp * rows_per + row;
    __syncthreads();  // thread 0 has seen the MMAs complete (the others wait here, idle)
    if (nkb > 0) {
      tc_fence_after();
      const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
      for (int c0 = 0; c0 < p.Mp; c0 += 64) {  // up to four loads in flight per wait
        uint32_t r[4][16];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 16 * u < p.Mp) tmem_ld16(t_row + static_cast<uint32_t>(c0 + 16 * u), r[u]);
        tmem_ld_wait();
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 16 * u < p.Mp) {
#pragma unroll
            for (int j = 0; j < 16; ++j) my[(c0 + 16 * u + j) * rows_per] = __uint_as_float(r[u][j]);
          }
      }
    } else {
      for (int m = 0; m < p.Mp; ++m) my[m * rows_per] = 0.f;
    }
    fence_proxy_async_shared();  // generic writes of send -> visible to the bulk copies
    __syncthreads();
    cluster_wait();  // every rank's recv_bar is initialised
    if (tid == 0) {
      const uint32_t src = smem_u32(send), dst = smem_u32(recv) + rank * slice_bytes,
                     bar = smem_u32(&recv_bar);
      for (int d = 0; d < p.split; ++d)
        bulk_to_peer(dsmem_map(dst, static_cast<uint32_t>(d)), src + static_cast<uint32_t>(d) * slice_bytes,
                     slice_bytes, dsmem_map(bar, static_cast<uint32_t>(d)));
    }
    if (tid == 0) ok_flag = mbar_wait(&recv_bar, 0, status) && ok_flag;
    __syncthreads();
    // Every slice sent TO this CTA has landed.  Arriving now (waiting only at
    // exit) keeps each CTA alive until all peers have received, i.e. until
    // every copy OUT of its send buffer is complete.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    // recv[src][m][row]: sum the split slices of rows [rank*rows_per, +rows_per)
    auto reduce_group = [&](int idx, const SkOps& o) {
      const int m = idx / g4, r4 = (idx % g4) * 4;
      const int n0 = tile * kSkTileN + static_cast<int>(rank) * rows_per + r4;
      if (n0 >= p.N) return;
      const float* base = recv + static_cast<size_t>(m) * rows_per + r4;
      float4 acc = *reinterpret_cast<const float4*>(base);
      for (int src = 1; src < p.split; ++src) {
        const float4 v = *reinterpret_cast<const float4*>(base + static_cast<size_t>(src) * p.Mp * rows_per);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      sk_store4(p, e, m, n0, acc, o);
    };
#pragma unroll
    for (int it = 0; it < kSkPre; ++it)
      if (tid + it * kSkThreads < total) reduce_group(tid + it * kSkThreads, pre[it]);
    for (int idx = tid + kSkPre * kSkThreads; idx < total; idx += kSkThreads) {
      const int m = idx / g4;
      const int n0 = tile * kSkTileN + static_cast<int>(rank) * rows_per + (idx % g4) * 4;
      reduce_group(idx, n0 < p.N ? sk_ops(p, e, m, n0)
                                 : SkOps{make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)});
    }
    cluster_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// K blocks one CTA can stage (a split > 1 also holds the receive buffer)
int sk_stage_cap(int mp, int split) {
  const int stage = kSkTileN * kSkBK * 2 + mp * kSkBK * 2;
  const int recv = split > 1 ? mp * kSkTileN * 4 : 0;
  return std::max(1, std::min(8, (kSkSmemBudget - recv) / stage));
}

}  // namespace

bool skinny_fits(long long M, long long N, long long K, long long ldx, long long ldw,
                 const void* x, const void* w) {
  if (M < 1 || M > kSkMaxM || N < 1 || N > 0x7fffffffLL || K < kSkBK || K % 8 || ldx % 8 ||
      ldw % 8)
    return false;
  if (!aligned16(x) || !aligned16(w)) return false;
  return true;  // any K: a CTA cycles its stage buffers as a ring
}

int skinny_run(const uint16_t* x, int M, long long ldx, const uint16_t* w, int N, long long ldw,
               int K, const TcEpilogue& e, cudaStream_t st, bool pdl, int force_split) {
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  if (!skinny_fits(M, N, K, ldx, ldw, x, w))
    return fail(GSVK_ERR_UNSUPPORTED, "skinny GEMM: M %d N %d K %d outside its range", M, N, K);
  SkProblem p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.Mp = (M + 15) / 16 * 16;
  p.kb_total = (K + kSkBK - 1) / kSkBK;
  const int stage_bytes = kSkTileN * kSkBK * 2 + p.Mp * kSkBK * 2;
  const int n_tiles = (N + kSkTileN - 1) / kSkTileN;
  // smallest power-of-two split that fits the stages, then widen while the
  // GPU is under-filled and every CTA still gets a K block
  // Split K only for up to 64 activation rows: the exchanged partial tile
  // grows with M (Mp x 128 fp32 per CTA), and from M = 65 up a whole-K CTA
  // per 128-row weight tile is cheaper than the cluster exchange.
  int split = 1;
  while (p.Mp <= 64 && split < kSkMaxSplit && static_cast<long long>(n_tiles) * split < sm_count() &&
         split * 2 <= p.kb_total)
    split *= 2;
  if (force_split > 0) {
    if (force_split > kSkMaxSplit || (force_split & (force_split - 1)) || force_split > p.kb_total)
      return fail(GSVK_ERR_INVALID, "skinny GEMM: split %d not usable for K %d", force_split, K);
    split = force_split;
  }
  p.split = split;
  p.stages = std::min((p.kb_total + split - 1) / split, sk_stage_cap(p.Mp, split));
  p.v_bias = e.bias && aligned16(e.bias);
  p.v_res = e.residual && aligned16(e.residual) && e.ld_res % 4 == 0;
  p.v_c32 = e.c32 && aligned16(e.c32) && e.ld_c32 % 4 == 0;
  p.v_c16 = e.c16 && (reinterpret_cast<uintptr_t>(e.c16) & 7u) == 0 && e.ld_c16 % 4 == 0;
  p.v_c16a = e.c16_act && (reinterpret_cast<uintptr_t>(e.c16_act) & 7u) == 0 && e.ld_c16_act % 4 == 0;
  const size_t tile_bytes = static_cast<size_t>(p.Mp) * kSkTileN * 4;
  const size_t smem = 1024 + (split > 1 ? tile_bytes : 0) +
                      std::max<size_t>(static_cast<size_t>(p.stages) * stage_bytes,
                                       split > 1 ? tile_bytes : 0);
  CUtensorMap tw, tx;
  int rc = make_kmajor_map(&tw, w, N, K, ldw, kSkTileN, kSkBK);
  if (!rc) rc = make_kmajor_map(&tx, x, M, K, ldx, p.Mp, kSkBK);
  if (rc) return rc;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    rc = check_cuda(cudaFuncSetAttribute(gemm_skinny_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSkSmemBudget + 2048),
                    "cudaFuncSetAttribute(gemm_skinny)");
    if (rc) return rc;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * split));
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (split > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = static_cast<unsigned>(split);
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return check_cuda(cudaLaunchKernelEx(&cfg, gemm_skinny_kernel, tw, tx, p, e, device_status()),
                    "gemm_skinny_kernel launch");
}

}  // namespace gsvk
