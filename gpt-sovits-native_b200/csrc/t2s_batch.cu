// t2s_batch.cu — batched T2S greedy decode: B concurrent utterances, each
// with its own KV cache and length (64 utterances,
// lengths U{64..1024}).
//
// One decode step streams every weight matrix once for all B tokens: the
// projections run as tensor-core GEMMs with M = B (gemm_tc.cuh, narrow
// 32-column tiles so that enough CTAs pull weights from HBM), the attention
// as split-KV chunks of 32 keys over each utterance's ragged cache, and
// sampling as one CTA per utterance (repetition penalty over its own
// history, 11-step EOS mask, t2s_engine.cpp:1594-1636).  The per-step
// positions come from a device step counter, so one captured CUDA graph
// replays every step.
//
// Numerics: fp16 operands with fp32 accumulation on the tensor cores (the
// W2 and logits activations are fp16 here, fp32 in the batch-1 path); parity
// with the oracle is at GEMM tolerance, not bit-exact.
#include <cmath>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_t2s_batch;

namespace gsvk {

namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 32;  // keys per attention CTA (split-KV)

struct BatchDev {
  int L, D, H, F, V, HD, cap, B, max_steps;
  float eps, alpha, scale;
  const uint16_t *wqkv, *wout, *w1, *w2, *wpred, *emb;
  const float *bqkv, *bout, *b1, *b2, *n1g, *n1b, *n2g, *n2b, *pe;
  uint16_t *kc, *vc;              // [B][L][cap][D]
  const int32_t* base_len;        // [B] slots filled before step 0
  const int32_t* base_pe;         // [B] PE index of step 0
  int32_t* step;                  // device step counter
  int32_t* tok;                   // [B] current input tokens
  uint8_t* seen;                  // [B][V] history marks
  int32_t* tokens_out;            // [max_steps][B]
  float* margins;                 // [max_steps][B] (optional)
};

__global__ void batch_embed_kernel(BatchDev m, float* __restrict__ x32, uint16_t* __restrict__ x16,
                                   int* __restrict__ attn_work) {
  const int b = blockIdx.x, D = m.D;
  const int s = *m.step;
  if (s >= m.max_steps) return;  // past the buffers: no-op
  griddep_launch_dependents();
  if (b == 0)  // the attention work counters of this step's layers
    for (int i = threadIdx.x; i < m.L; i += blockDim.x) attn_work[i] = 0;
  const uint16_t* er = m.emb + static_cast<size_t>(m.tok[b]) * D;
  const float* pr = m.pe + static_cast<size_t>(m.base_pe[b] + s) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = fmaf(m.alpha, pr[i], h2f(er[i]));
    x32[static_cast<size_t>(b) * D + i] = v;
    x16[static_cast<size_t>(b) * D + i] = f2h(v);
  }
}

// Split-KV one-query attention (flash-decoding).  CTA (c, b) takes keys
// [32c, 32c + 32) of utterance b for ALL heads: the chunk's K and V rows are
// contiguous in the [b][L][cap][D] cache, so two 1D bulk copies bring them
// into shared memory at full HBM efficiency.  A warp reads 256 halves of a
// row (16 bytes per lane, conflict-free); lanes sharing a head reduce with
// shuffles.  The chunk that holds the new slot (base_len[b] + step) appends
// the step's K/V row to the cache and to its shared copy.  Each chunk writes
// (max, sum, unnormalised output) per head; the chunk that takes the last
// ticket of its utterance merges them — no CTA waits on another.
__global__ void __launch_bounds__(kAttnThreads) batch_attn_kernel(BatchDev m, int l,
                                                                  const float* __restrict__ qkv,
                                                                  uint16_t* __restrict__ out16,
                                                                  float* __restrict__ part_o,
                                                                  float2* __restrict__ part_ml,
                                                                  unsigned* __restrict__ ticket,
                                                                  int max_chunks,
                                                                  uint32_t* status) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  __shared__ uint64_t bars[2];
  __shared__ int is_last;
  const int D = m.D, H = m.H, HD = m.HD;
  const int b = blockIdx.y, c = blockIdx.x;
  const int s = *m.step;
  if (s >= m.max_steps) return;
  const int pos = m.base_len[b] + s;
  const int len = pos + 1;
  const int nchunks = (len + kAttnChunk - 1) / kAttnChunk;
  if (c >= nchunks) return;
  const int k0 = c * kAttnChunk;
  const int rows = min(kAttnChunk, len - k0);
  uint16_t* sK = reinterpret_cast<uint16_t*>(attn_smem);
  uint16_t* sV = sK + kAttnChunk * D;
  float* sP = reinterpret_cast<float*>(sV + kAttnChunk * D);  // [H][kAttnChunk + 1]
  float* sM = sP + H * (kAttnChunk + 1);
  float* sL = sM + H;
  float* sPart = reinterpret_cast<float*>(sK);  // PV partials reuse the K buffer
  const size_t slab = (static_cast<size_t>(b) * m.L + l) * m.cap + k0;
  uint16_t* kg = m.kc + slab * D;
  uint16_t* vg = m.vc + slab * D;
  const float* qrow = qkv + static_cast<size_t>(b) * 3 * D;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
    const uint32_t bytes = static_cast<uint32_t>(rows) * D * 2;
    mbar_arrive_expect_tx(&bars[0], bytes);
    bulk_load(sK, kg, bytes, &bars[0]);
    mbar_arrive_expect_tx(&bars[1], bytes);
    bulk_load(sV, vg, bytes, &bars[1]);
  }
  griddep_wait();  // q and the new K/V row come from the QKV projection
  griddep_launch_dependents();
  // lane geometry: a warp covers segment `seg` (256 halves) of rows rg, rg + nrg, ...
  const int nseg = D / 256, nrg = (kAttnThreads / 32) / nseg;
  const int seg = warp % nseg, rg = warp / nseg;
  const int e0 = seg * 256 + lane * 8;
  const int lph = HD / 8, head = e0 / HD;
  float q[8];
  {
    const float4 q0 = *reinterpret_cast<const float4*>(qrow + e0);
    const float4 q1 = *reinterpret_cast<const float4*>(qrow + e0 + 4);
    q[0] = q0.x * m.scale; q[1] = q0.y * m.scale; q[2] = q0.z * m.scale; q[3] = q0.w * m.scale;
    q[4] = q1.x * m.scale; q[5] = q1.y * m.scale; q[6] = q1.z * m.scale; q[7] = q1.w * m.scale;
  }
  // the new slot pos = len - 1 is row rows - 1 of the last chunk; no other chunk touches it
  const int r_new = (c == nchunks - 1) ? rows - 1 : -1;
  __syncthreads();
  if (!__syncthreads_and(mbar_wait(&bars[0], 0, status))) return;
  if (r_new >= 0) {
    for (int i = tid; i < D; i += kAttnThreads) {
      const uint16_t kv = f2h(qrow[D + i]);
      sK[r_new * D + i] = kv;
      kg[static_cast<size_t>(r_new) * D + i] = kv;
    }
    __syncthreads();
  }
  for (int r = rg; r < rows; r += nrg) {
    float kf[8];
    unpack8(*reinterpret_cast<const uint4*>(sK + r * D + e0), kf);
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) d = fmaf(q[j], kf[j], d);
    for (int o = 1; o < lph; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if ((lane & (lph - 1)) == 0) sP[head * (kAttnChunk + 1) + r] = d;
  }
  __syncthreads();
  for (int h = warp; h < H; h += kAttnThreads / 32) {
    float* ph = sP + h * (kAttnChunk + 1);
    float mx = -INFINITY;
    for (int r = lane; r < rows; r += 32) mx = fmaxf(mx, ph[r]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int r = lane; r < rows; r += 32) {
      const float p = expf(ph[r] - mx);
      ph[r] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      sM[h] = mx;
      sL[h] = sum;
    }
  }
  if (!__syncthreads_and(mbar_wait(&bars[1], 0, status))) return;
  if (r_new >= 0) {
    for (int i = tid; i < D; i += kAttnThreads) {
      const uint16_t vv = f2h(qrow[2 * D + i]);
      sV[r_new * D + i] = vv;
      vg[static_cast<size_t>(r_new) * D + i] = vv;
    }
    __syncthreads();
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r = rg; r < rows; r += nrg) {
    const float p = sP[head * (kAttnChunk + 1) + r];
    float vf[8];
    unpack8(*reinterpret_cast<const uint4*>(sV + r * D + e0), vf);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = fmaf(p, vf[j], acc[j]);
  }
  float4* pw = reinterpret_cast<float4*>(sPart + warp * 256 + lane * 8);
  pw[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  pw[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  __syncthreads();
  const size_t pc = static_cast<size_t>(b) * max_chunks;
  for (int i = tid; i < D; i += kAttnThreads) {
    const int sg = i >> 8, w = i & 255;
    float o = 0.f;
    for (int g = 0; g < nrg; ++g) o += sPart[(g * nseg + sg) * 256 + w];
    if (nchunks == 1)
      out16[static_cast<size_t>(b) * D + i] = f2h(o / sL[i / HD]);
    else
      part_o[(pc + c) * D + i] = o;
  }
  if (nchunks == 1) return;
  if (tid < H) part_ml[(pc + c) * H + tid] = make_float2(sM[tid], sL[tid]);
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&ticket[b], 1u) == static_cast<unsigned>(nchunks - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // merge: out = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c, per head
  if (tid < H) {
    float M = -INFINITY;
    for (int cc = 0; cc < nchunks; ++cc) M = fmaxf(M, __ldcg(&part_ml[(pc + cc) * H + tid]).x);
    float den = 0.f;
    for (int cc = 0; cc < nchunks; ++cc) {
      const float2 ml = __ldcg(&part_ml[(pc + cc) * H + tid]);
      den = fmaf(expf(ml.x - M), ml.y, den);
    }
    sM[tid] = M;
    sL[tid] = den;
  }
  __syncthreads();
  for (int i = tid; i < D; i += kAttnThreads) {
    const int h = i / HD;
    const float M = sM[h];
    float num = 0.f;
    for (int cc = 0; cc < nchunks; ++cc)
      num = fmaf(expf(__ldcg(&part_ml[(pc + cc) * H + h]).x - M), __ldcg(&part_o[(pc + cc) * D + i]),
                 num);
    out16[static_cast<size_t>(b) * D + i] = f2h(num / sL[h]);
  }
  if (tid == 0) ticket[b] = 0;
}

// Streaming split-KV attention (d_model <= 512): one persistent CTA per SM
// walks work items (utterance b, split sp) = keys [kAttnSplitKeys*sp,
// +kAttnSplitKeys) of b, all heads.  Thread 0 keeps kAttnStages chunk
// copies (16 keys of K and of V, two 1D bulk copies) in flight across items:
// each CTA's first item is fixed (its block index), later ones come from a
// per-layer work counter (zeroed by the step's embedding kernel).  Items are
// handed out longest first: every full split (kAttnSplitChunks chunks), then
// each utterance's shorter last split by decreasing length, so the CTAs that
// take a second item take short ones and finish together.  Within an
// item the softmax runs online over its chunks (running max / sum per head,
// accumulator rescaled); a one-split utterance writes its output directly,
// otherwise each split writes (max, sum, unnormalised output) per head and the
// split that takes the utterance's last ticket merges them.
constexpr int kAttnStages = 3;
constexpr int kSChunk = 16;  // keys per streamed chunk (two CTAs per SM)
constexpr int kAttnSplitChunks = 8;
constexpr int kAttnSplitKeys = kSChunk * kAttnSplitChunks;

size_t attn_stream_smem_bytes(int D, int H, int B) {
  return static_cast<size_t>(kAttnStages) * kSChunk * D * 2 * 2 +  // K, V ring
         static_cast<size_t>(kAttnThreads / 32) * 256 * 4 +            // PV partials
         (static_cast<size_t>(H) * (kSChunk + 1) + 4 * H) * 4 +     // P, max/sum/scale
         static_cast<size_t>(4 * B + 2 + 3 * kAttnStages) * 4 + 64;    // item offsets, lengths, order, slots
}

template <int NSEG>
__global__ void __launch_bounds__(kAttnThreads, 2)
    batch_attn_stream_kernel(BatchDev m, int l, const float* __restrict__ qkv,
                             uint16_t* __restrict__ out16, float* __restrict__ part_o,
                             float2* __restrict__ part_ml, unsigned* __restrict__ ticket,
                             int* __restrict__ work, int max_chunks, uint32_t* status) {
  extern __shared__ __align__(128) uint8_t as_smem[];
  __shared__ uint64_t full[kAttnStages];
  __shared__ int is_last;
  const int D = m.D, H = m.H, HD = m.HD, B = m.B;
  const int s = *m.step;
  if (s >= m.max_steps) return;
  uint16_t* kbuf = reinterpret_cast<uint16_t*>(as_smem);
  uint16_t* vbuf = kbuf + static_cast<size_t>(kAttnStages) * kSChunk * D;
  float* sPart = reinterpret_cast<float*>(vbuf + static_cast<size_t>(kAttnStages) * kSChunk * D);
  float* sP = sPart + (kAttnThreads / 32) * 256;  // [H][kSChunk + 1]
  float* sMr = sP + H * (kSChunk + 1);          // running max per head
  float* sLr = sMr + H;                            // running sum per head
  float* sSc = sLr + H;                            // this chunk's rescale of the accumulator
  int* sOff = reinterpret_cast<int*>(sSc + H);     // [B + 1] first item of each utterance
  int* sItem = sOff + B + 1;                       // [kAttnStages] item of the slot's chunk (-1: none)
  int* sChunk = sItem + kAttnStages;               // [kAttnStages] chunk index in its utterance
  int* sLen = sChunk + kAttnStages;                // [B] keys of each utterance this step (the
                                                   // per-chunk paths read it, not global memory)
  int* sFull = sLen + B;                           // [B + 1] first full split of each utterance,
                                                   // in dispatch order
  int* sShort = sFull + B + 1;                     // [B] utterances with a short last split,
                                                   // longest first
  int* sUtt = sShort + B;                          // [kAttnStages] utterance of the slot's chunk
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    for (int i = 0; i < kAttnStages; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
    int acc = 0, full = 0;
    for (int b = 0; b < B; ++b) {
      const int len = m.base_len[b] + s + 1;
      sLen[b] = len;
      sOff[b] = acc;
      sFull[b] = full;
      acc += (len + kAttnSplitKeys - 1) / kAttnSplitKeys;
      full += len / kAttnSplitKeys;
    }
    sOff[B] = acc;
    sFull[B] = full;
  }
  __syncthreads();
  const int n_items = sOff[B], n_full = sFull[B];
  // rank of each short last split: longer first, then by utterance
  for (int b = tid; b < B; b += kAttnThreads) {
    const int rb = sLen[b] % kAttnSplitKeys;
    if (rb == 0) continue;
    int rank = 0;
    for (int o = 0; o < B; ++o) {
      const int ro = sLen[o] % kAttnSplitKeys;
      rank += (ro > rb || (ro == rb && o < b)) ? 1 : 0;
    }
    sShort[rank] = b;
  }
  __syncthreads();
  auto item_utt = [&](int it) {  // the utterance of item `it` (binary search)
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sOff[mid] <= it) lo = mid; else hi = mid - 1;
    }
    return lo;
  };
  // the item handed out d-th: full splits in utterance order, then the short
  // last splits as ranked above
  auto dispatch_item = [&](int d) {
    if (d >= n_full) {
      const int b = sShort[d - n_full];
      return sOff[b + 1] - 1;
    }
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sFull[mid] <= d) lo = mid; else hi = mid - 1;
    }
    return sOff[lo] + (d - sFull[lo]);
  };
  // ---- producer (thread 0): the CTA's chunk sequence, one slot at a time
  int p_item = -1, p_b = 0, p_c = 0, p_cend = 0, p_grab = 0, p_n = 0;
  bool p_done = false;
  auto produce = [&](bool dynamic) -> bool {  // false: nothing issued (needs the work counter)
    const int sl = p_n % kAttnStages;
    while (!p_done && p_c >= p_cend) {  // next item
      int it;
      if (p_grab == 0) {
        it = blockIdx.x;
      } else {
        if (!dynamic) return false;
        it = static_cast<int>(gridDim.x) + atomicAdd(work + l, 1);
      }
      ++p_grab;
      if (it >= n_items) {
        p_done = true;
        break;
      }
      it = dispatch_item(it);
      const int b = item_utt(it), sp = it - sOff[b];
      const int nch = (sLen[b] + kSChunk - 1) / kSChunk;
      p_item = it;
      p_b = b;
      p_c = sp * kAttnSplitChunks;
      p_cend = min(nch, p_c + kAttnSplitChunks);
    }
    if (p_done) {
      sItem[sl] = -1;
      mbar_arrive(&full[sl]);  // completes the phase with no copy: the consumers stop here
    } else {
      const int b = p_b;
      const int len = sLen[b];
      const int k0 = p_c * kSChunk, rows = min(kSChunk, len - k0);
      const size_t slab = (static_cast<size_t>(b) * m.L + l) * m.cap + k0;
      const uint32_t bytes = static_cast<uint32_t>(rows) * D * 2;
      sItem[sl] = p_item;
      sUtt[sl] = p_b;
      sChunk[sl] = p_c;
      mbar_arrive_expect_tx(&full[sl], 2 * bytes);
      bulk_load(kbuf + static_cast<size_t>(sl) * kSChunk * D, m.kc + slab * D, bytes, &full[sl]);
      bulk_load(vbuf + static_cast<size_t>(sl) * kSChunk * D, m.vc + slab * D, bytes, &full[sl]);
      ++p_c;
    }
    ++p_n;
    return true;
  };
  if (tid == 0) {  // the fixed first item's chunks, before the dependency resolves
    while (p_n < kAttnStages && produce(false)) {
    }
  }
  griddep_wait();  // q and the new K/V rows come from the QKV projection
  griddep_launch_dependents();
  if (tid == 0) {
    while (p_n < kAttnStages) produce(true);
  }
  // lane geometry: a warp covers segment `seg` (256 halves) of rows rg, rg + nrg, ...
  constexpr int nrg = (kAttnThreads / 32) / NSEG;  // row groups
  constexpr int kRows = kSChunk / nrg;          // rows per warp and chunk
  const int seg = warp % NSEG, rg = warp / NSEG;
  const int e0 = seg * 256 + lane * 8;
  const int lph = HD / 8, head = e0 / HD;
  float q[8], acc[8];
  bool failed = false;
  for (uint32_t ci = 0;; ++ci) {
    const int sl = static_cast<int>(ci % kAttnStages);
    // one lane per warp polls; the rest park at the warp barrier
    if (!failed) {
      bool ok = true;
      if (lane == 0) {
        ok = false;
        for (uint32_t i = 0; i < kSpinLimit && !ok; ++i) ok = mbar_try_wait(&full[sl], (ci / kAttnStages) & 1u);
        if (!ok) atomicExch(status, DEV_TIMEOUT);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (ok) mbar_try_wait(&full[sl], (ci / kAttnStages) & 1u);  // this lane's acquire
      failed = !ok;
    }
    if (!__syncthreads_and(!failed)) break;
    const int it = sItem[sl];
    if (it < 0) break;
    const int c = sChunk[sl];
    const int b = sUtt[sl], sp = it - sOff[b];
    const int len = sLen[b];
    const int nch = (len + kSChunk - 1) / kSChunk;
    const int nsplit = sOff[b + 1] - sOff[b];
    const int k0 = c * kSChunk, rows = min(kSChunk, len - k0);
    const bool first = c == sp * kAttnSplitChunks;
    const bool last = c == min(nch, (sp + 1) * kAttnSplitChunks) - 1;
    uint16_t* sK = kbuf + static_cast<size_t>(sl) * kSChunk * D;
    uint16_t* sV = vbuf + static_cast<size_t>(sl) * kSChunk * D;
    const float* qrow = qkv + static_cast<size_t>(b) * 3 * D;
    if (first) {  // a new item: its query and a fresh running state
      const float4 q0 = *reinterpret_cast<const float4*>(qrow + e0);
      const float4 q1 = *reinterpret_cast<const float4*>(qrow + e0 + 4);
      q[0] = q0.x * m.scale; q[1] = q0.y * m.scale; q[2] = q0.z * m.scale; q[3] = q0.w * m.scale;
      q[4] = q1.x * m.scale; q[5] = q1.y * m.scale; q[6] = q1.z * m.scale; q[7] = q1.w * m.scale;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      if (tid < H) {
        sMr[tid] = -INFINITY;
        sLr[tid] = 0.f;
      }
    }
    if (c == nch - 1) {  // the new slot pos = len - 1: append this step's K / V row
      const size_t slab = (static_cast<size_t>(b) * m.L + l) * m.cap + k0;
      const int r_new = rows - 1;
      for (int i = tid; i < D; i += kAttnThreads) {
        const uint16_t kv = f2h(qrow[D + i]), vv = f2h(qrow[2 * D + i]);
        sK[r_new * D + i] = kv;
        sV[r_new * D + i] = vv;
        m.kc[(slab + r_new) * D + i] = kv;
        m.vc[(slab + r_new) * D + i] = vv;
      }
    }
    __syncthreads();
    {  // scores of this warp's kRows rows: all loads first, independent chains
      uint4 kr[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = rg + i * nrg;
        kr[i] = r < rows ? *reinterpret_cast<const uint4*>(sK + r * D + e0) : make_uint4(0, 0, 0, 0);
      }
      float d[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        float kf[8];
        unpack8(kr[i], kf);
        d[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) d[i] = fmaf(q[j], kf[j], d[i]);
      }
      for (int o = 1; o < lph; o <<= 1) {
#pragma unroll
        for (int i = 0; i < kRows; ++i) d[i] += __shfl_xor_sync(0xffffffffu, d[i], o);
      }
      if ((lane & (lph - 1)) == 0) {
#pragma unroll
        for (int i = 0; i < kRows; ++i) {
          const int r = rg + i * nrg;
          if (r < rows) sP[head * (kSChunk + 1) + r] = d[i];
        }
      }
    }
    __syncthreads();
    {  // online softmax: lanes 0-15 take head `warp`, lanes 16-31 head
       // `warp + 8`, one key per lane (the sums are the same butterflies)
      static_assert(kSChunk == 16, "one key per half-warp lane");
      const int hh = warp + (lane >> 4) * (kAttnThreads / 32), r = lane & 15;
      const bool ok = hh < H, in = ok && r < rows;
      float* ph = sP + (ok ? hh : 0) * (kSChunk + 1);
      const float sv = in ? ph[r] : -INFINITY;
      const float mx0 = warp_max(lane < 16 ? sv : -INFINITY);
      const float mx1 = warp_max(lane < 16 ? -INFINITY : sv);
      const float mo = ok ? sMr[hh] : 0.f;
      const float mn = fmaxf(mo, lane < 16 ? mx0 : mx1);
      const float ev = in ? expf(sv - mn) : 0.f;
      if (in) ph[r] = ev;
      float su = ev;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) su += __shfl_xor_sync(0xffffffffu, su, o);
      if (r == 0 && ok) {
        const float sc = mo == -INFINITY ? 0.f : expf(mo - mn);
        sSc[hh] = sc;
        sLr[hh] = fmaf(sLr[hh], sc, su);
        sMr[hh] = mn;
      }
    }
    __syncthreads();
    {  // P.V of this warp's rows: all loads first
      uint4 vr[kRows];
      float pr[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = rg + i * nrg;
        const bool ok = r < rows;
        vr[i] = ok ? *reinterpret_cast<const uint4*>(sV + r * D + e0) : make_uint4(0, 0, 0, 0);
        pr[i] = ok ? sP[head * (kSChunk + 1) + r] : 0.f;
      }
      const float sc = sSc[head];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] *= sc;
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        float vf[8];
        unpack8(vr[i], vf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(pr[i], vf[j], acc[j]);
      }
    }
    __syncthreads();  // every thread is done with the slot
    if (tid == 0) produce(true);
    if (!last) continue;
    // ---- the item is complete: reduce the row groups, then output / partial
    float4* pw = reinterpret_cast<float4*>(sPart + warp * 256 + lane * 8);
    pw[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    pw[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    __syncthreads();
    const size_t pc = static_cast<size_t>(b) * max_chunks;
    for (int i = tid; i < D; i += kAttnThreads) {
      const int sg = i >> 8, w = i & 255;
      float o = 0.f;
      for (int g = 0; g < nrg; ++g) o += sPart[(g * NSEG + sg) * 256 + w];
      if (nsplit == 1)
        out16[static_cast<size_t>(b) * D + i] = f2h(o / sLr[i / HD]);
      else
        part_o[(pc + sp) * D + i] = o;
    }
    if (nsplit > 1) {
      if (tid < H) part_ml[(pc + sp) * H + tid] = make_float2(sMr[tid], sLr[tid]);
      __threadfence();
      __syncthreads();
      if (tid == 0) is_last = atomicAdd(&ticket[b], 1u) == static_cast<unsigned>(nsplit - 1);
      __syncthreads();
      if (is_last) {
        __threadfence();
        // out = sum_sp e^(m_sp - M) o_sp / sum_sp e^(m_sp - M) l_sp, per head
        if (tid < H) {
          float M = -INFINITY;
          for (int cc = 0; cc < nsplit; ++cc) M = fmaxf(M, __ldcg(&part_ml[(pc + cc) * H + tid]).x);
          float den = 0.f;
          for (int cc = 0; cc < nsplit; ++cc) {
            const float2 ml = __ldcg(&part_ml[(pc + cc) * H + tid]);
            den = fmaf(expf(ml.x - M), ml.y, den);
          }
          sSc[tid] = M;
          sP[tid] = den;
        }
        __syncthreads();
        for (int i = tid; i < D; i += kAttnThreads) {
          const int h = i / HD;
          const float M = sSc[h];
          float num = 0.f;
          for (int cc = 0; cc < nsplit; ++cc)
            num = fmaf(expf(__ldcg(&part_ml[(pc + cc) * H + h]).x - M),
                       __ldcg(&part_o[(pc + cc) * D + i]), num);
          out16[static_cast<size_t>(b) * D + i] = f2h(num / sP[h]);
        }
        if (tid == 0) ticket[b] = 0;
      }
    }
    __syncthreads();  // sPart / sP / sSc are reused by the next item
  }
}

size_t attn_smem_bytes(int D, int H) {
  return static_cast<size_t>(kAttnChunk) * D * 2 * 2 +
         (static_cast<size_t>(H) * (kAttnChunk + 1) + 2 * H) * 4;
}

__global__ void batch_ln_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                const float* __restrict__ bta, float* __restrict__ y,
                                uint16_t* __restrict__ y16, int n, double eps) {
  __shared__ double sh[64];
  griddep_wait();
  griddep_launch_dependents();
  const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
  float s = 0.f, q = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i];
    s += v;
    q = fmaf(v, v, q);
  }
  double ds = warp_sum_d(static_cast<double>(s)), dq = warp_sum_d(static_cast<double>(q));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sh[w] = ds;
    sh[32 + w] = dq;
  }
  __syncthreads();
  ds = lane < nw ? sh[lane] : 0.0;
  dq = lane < nw ? sh[32 + lane] : 0.0;
  ds = warp_sum_d(ds);
  dq = warp_sum_d(dq);
  const float mean = static_cast<float>(ds / n);
  float var = static_cast<float>(dq / n - static_cast<double>(mean) * mean);
  if (!(var >= 0.f)) var = 0.f;
  const float rstd = static_cast<float>(1.0 / sqrt(static_cast<double>(var) + eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = fmaf((xr[i] - mean) * rstd, g[i], bta[i]);
    y[static_cast<size_t>(blockIdx.x) * n + i] = v;
    y16[static_cast<size_t>(blockIdx.x) * n + i] = f2h(v);
  }
}

// Greedy sample of utterance b (penalty 1.35 once per distinct history
// token, EOS excluded while step < 11), then advance: record the token, mark
// it seen, make it the next input.  The last block bumps the step counter.
__global__ void batch_sample_kernel(BatchDev m, const float* __restrict__ logits,
                                    unsigned* __restrict__ done) {
  __shared__ float rv[32];
  __shared__ float rs[32];
  __shared__ int ri[32];
  const int b = blockIdx.x, V = m.V;
  griddep_wait();
  const int s = *m.step;
  if (s >= m.max_steps) return;
  const int limit = s >= 11 ? V : V - 1;
  const float* lg = logits + static_cast<size_t>(b) * V;
  const uint8_t* seen = m.seen + static_cast<size_t>(b) * V;
  float bv = -INFINITY, sv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < limit; c += blockDim.x) {
    float v = lg[c];
    if (seen[c]) v = v < 0.f ? v * 1.35f : v / 1.35f;
    if (v > bv || (v == bv && c < bi)) {
      sv = bv;
      bv = v;
      bi = c;
    } else if (v > sv) {
      sv = v;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o), os = __shfl_xor_sync(0xffffffffu, sv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      sv = fmaxf(os, bv);
      bv = ov;
      bi = oi;
    } else {
      sv = fmaxf(sv, ov);
    }
  }
  if (lane == 0) {
    rv[w] = bv;
    rs[w] = sv;
    ri[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float B = rv[0], S = rs[0];
    int I = ri[0];
    for (int k = 1; k < nw; ++k) {
      if (rv[k] > B || (rv[k] == B && ri[k] < I)) {
        S = fmaxf(rs[k], B);
        B = rv[k];
        I = ri[k];
      } else {
        S = fmaxf(S, rv[k]);
      }
    }
    m.tokens_out[static_cast<size_t>(s) * m.B + b] = I;
    if (m.margins) m.margins[static_cast<size_t>(s) * m.B + b] = B - S;
    m.seen[static_cast<size_t>(b) * V + I] = 1;
    m.tok[b] = I;
    __threadfence();
    if (atomicAdd(done, 1u) == static_cast<unsigned>(m.B) - 1) {
      *done = 0;
      *m.step = s + 1;
    }
  }
}

}  // namespace

struct T2SBatchEngine {
  BatchDev d{};
  int max_batch = 0, cur_batch = 0;
  void* wmem = nullptr;
  void* amem = nullptr;
  int32_t *base_len = nullptr, *base_pe = nullptr, *step = nullptr, *tok = nullptr,
          *tokens_out = nullptr;
  float* margins = nullptr;
  unsigned* done = nullptr;
  unsigned* ticket = nullptr;  // [B] attention merge tickets (zero between launches)
  int* attn_work = nullptr;    // [L] streaming attention work counters (zeroed per step)
  bool attn_stream = false;    // the streaming attention kernel (d_model <= 512)
  int attn_kind = 0;           // 0 per-chunk CTAs, 1 streaming CTAs
  float* part_o = nullptr;     // [B][max_chunks][D] per-chunk attention outputs
  float2* part_ml = nullptr;   // [B][max_chunks][H] per-chunk (max, sum)
  int max_chunks = 0;
  uint8_t* seen = nullptr;
  float *x32 = nullptr, *qkv32 = nullptr, *hpre32 = nullptr, *h32 = nullptr, *xpre32 = nullptr,
        *logits = nullptr;
  uint16_t *x16 = nullptr, *attn16 = nullptr, *h16 = nullptr, *ff16 = nullptr;
  int max_steps = 0;
  int host_step = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int graph_batch = 0;
  int launches_per_step = 0;
};

namespace {

int gemm_m(const uint16_t* A, int M, int K, const uint16_t* W, int N, const float* bias, int act,
           const float* res, float* c32, uint16_t* c16, cudaStream_t st) {
  TcProblem p{};
  p.M = M;
  p.N = N;
  p.kc = K;
  p.taps = 1;
  p.dil = 1;
  p.phases = 1;
  p.out_rows = M;
  TcEpilogue e = make_epilogue();
  e.bias = bias;
  e.act = act;
  e.residual = res;
  e.ld_res = N;
  e.c32 = c32;
  e.ld_c32 = N;
  e.c16 = c16;
  e.ld_c16 = N;
  if (skinny_fits(M, N, K, K, K, A, W)) return skinny_run(A, M, K, W, N, K, K, e, st, true);
  // 32-column tiles: N/32 CTAs stream the weight matrix
  return tc_run(A, M, K, W, N, K, p, e, 32, st);
}

int batch_step(T2SBatchEngine* e, int B, cudaStream_t st, int* launches) {
  BatchDev& m = e->d;
  const int D = m.D, F = m.F;
  int n = 0, rc;
  batch_embed_kernel<<<B, 256, 0, st>>>(m, e->x32, e->x16, e->attn_work);
  if ((rc = check_launch("batch_embed_kernel"))) return rc;
  ++n;
  for (int l = 0; l < m.L; ++l) {
    if ((rc = gemm_m(e->x16, B, D, m.wqkv + (size_t)l * 3 * D * D, 3 * D,
                     m.bqkv + (size_t)l * 3 * D, GSVK_ACT_NONE, nullptr, e->qkv32, nullptr, st)))
      return rc;
    if (e->attn_kind == 1) {
      auto* fn = D == 512 ? batch_attn_stream_kernel<2> : batch_attn_stream_kernel<1>;
      if ((rc = launch_pdl(fn, dim3(2 * sm_count()), dim3(kAttnThreads),
                           attn_stream_smem_bytes(D, m.H, m.B), st, "batch_attn_stream_kernel", m,
                           l, e->qkv32, e->attn16, e->part_o, e->part_ml, e->ticket, e->attn_work,
                           e->max_chunks, device_status())))
        return rc;
    } else if ((rc = launch_pdl(batch_attn_kernel, dim3(e->max_chunks, B), dim3(kAttnThreads),
                                attn_smem_bytes(D, m.H), st, "batch_attn_kernel", m, l, e->qkv32,
                                e->attn16, e->part_o, e->part_ml, e->ticket, e->max_chunks,
                                device_status()))) {
      return rc;
    }
    if ((rc = gemm_m(e->attn16, B, D, m.wout + (size_t)l * D * D, D, m.bout + (size_t)l * D,
                     GSVK_ACT_NONE, e->x32, e->hpre32, nullptr, st)))
      return rc;
    if ((rc = launch_pdl(batch_ln_kernel, dim3(B), dim3(256), 0, st, "batch_ln_kernel", e->hpre32,
                         m.n1g + (size_t)l * D, m.n1b + (size_t)l * D, e->h32, e->h16, D,
                         static_cast<double>(m.eps))))
      return rc;
    if ((rc = gemm_m(e->h16, B, D, m.w1 + (size_t)l * F * D, F, m.b1 + (size_t)l * F,
                     GSVK_ACT_RELU, nullptr, nullptr, e->ff16, st)))
      return rc;
    if ((rc = gemm_m(e->ff16, B, F, m.w2 + (size_t)l * D * F, D, m.b2 + (size_t)l * D,
                     GSVK_ACT_NONE, e->h32, e->xpre32, nullptr, st)))
      return rc;
    if ((rc = launch_pdl(batch_ln_kernel, dim3(B), dim3(256), 0, st, "batch_ln_kernel", e->xpre32,
                         m.n2g + (size_t)l * D, m.n2b + (size_t)l * D, e->x32, e->x16, D,
                         static_cast<double>(m.eps))))
      return rc;
    n += 7;
  }
  if ((rc = gemm_m(e->x16, B, D, m.wpred, m.V, nullptr, GSVK_ACT_NONE, nullptr, e->logits,
                   nullptr, st)))
    return rc;
  if ((rc = launch_pdl(batch_sample_kernel, dim3(B), dim3(256), 0, st, "batch_sample_kernel", m,
                       e->logits, e->done)))
    return rc;
  n += 2;
  if (launches) *launches = n;
  return GSVK_OK;
}

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

void pe_rows(int D, int cap, float* pe) {
  const float log_inc = static_cast<float>(-std::log(10000.0) / static_cast<double>(D));
  for (int p = 0; p < cap; ++p) {
    const float pf = static_cast<float>(p);
    for (int d = 0; d < D; d += 2) {
      const float div = std::exp(static_cast<float>(d) * log_inc);
      pe[(size_t)p * D + d] = std::sin(pf * div);
      pe[(size_t)p * D + d + 1] = std::cos(pf * div);
    }
  }
}

}  // namespace
}  // namespace gsvk

using namespace gsvk;

struct gsvk_t2s_batch : gsvk::T2SBatchEngine {};

extern "C" {

int gsvk_t2s_batch_destroy(gsvk_t2s_batch_t h) {
  if (!h) return GSVK_OK;
  if (h->exec) cudaGraphExecDestroy(h->exec);
  if (h->graph) cudaGraphDestroy(h->graph);
  if (h->wmem) cudaFree(h->wmem);
  if (h->amem) cudaFree(h->amem);
  delete h;
  return GSVK_OK;
}

int gsvk_t2s_batch_create(const gsvk_t2s_config* cfg, const gsvk_t2s_host_weights* w,
                          int max_batch, int max_steps, gsvk_t2s_batch_t* out) {
  if (!cfg || !w || !out) return fail(GSVK_ERR_INVALID, "t2s_batch_create: null argument");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  const int L = cfg->n_layers, D = cfg->d_model, H = cfg->n_heads, F = cfg->ffn, V = cfg->vocab;
  const int cap = cfg->cap;
  if (L <= 0 || D <= 0 || H <= 0 || F <= 0 || V <= 1 || cap <= 0 || D % H || max_batch <= 0 ||
      max_batch > 128 || max_steps <= 0)
    return fail(GSVK_ERR_INVALID, "t2s_batch_create: bad dimensions");
  const int HD = D / H;
  if ((HD != 32 && HD != 64) || (D != 256 && D != 512 && D != 1024 && D != 2048) || F % 64)
    return fail(GSVK_ERR_UNSUPPORTED,
                "t2s_batch_create: head_dim 32/64, d_model 256/512/1024/2048, ffn multiple of 64");
  if (attn_smem_bytes(D, H) > 200 * 1024)
    return fail(GSVK_ERR_UNSUPPORTED, "t2s_batch_create: attention chunk exceeds shared memory");
  if (!w->wqkv || !w->bqkv || !w->wout || !w->bout || !w->w1 || !w->b1 || !w->w2 || !w->b2 ||
      !w->n1g || !w->n1b || !w->n2g || !w->n2b || !w->wpred || !w->audio_emb)
    return fail(GSVK_ERR_INVALID, "t2s_batch_create: null weight");
  auto* e = new gsvk_t2s_batch();
  e->max_batch = max_batch;
  e->max_steps = max_steps;
  BatchDev& d = e->d;
  d.max_steps = max_steps;
  d.L = L; d.D = D; d.H = H; d.F = F; d.V = V; d.HD = HD; d.cap = cap;
  d.eps = cfg->ln_eps; d.alpha = cfg->alpha_audio;
  d.scale = 1.0f / std::sqrt(static_cast<float>(HD));
  const size_t nq = (size_t)L * 3 * D * D, no = (size_t)L * D * D, n1 = (size_t)L * F * D,
               n2 = (size_t)L * D * F, np = (size_t)V * D;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al256(bytes); return o; };
  struct Up { size_t o; const void* src; size_t bytes; };
  std::vector<Up> ups;
  auto up = [&](const void* src, size_t bytes) { ups.push_back({take(bytes), src, bytes}); return ups.back().o; };
  std::vector<float> pe((size_t)cap * D);
  pe_rows(D, cap, pe.data());
  const size_t o_q = up(w->wqkv, nq * 2), o_o = up(w->wout, no * 2), o_1 = up(w->w1, n1 * 2),
               o_2 = up(w->w2, n2 * 2), o_p = up(w->wpred, np * 2), o_e = up(w->audio_emb, np * 2),
               o_bq = up(w->bqkv, (size_t)L * 3 * D * 4), o_bo = up(w->bout, (size_t)L * D * 4),
               o_b1 = up(w->b1, (size_t)L * F * 4), o_b2 = up(w->b2, (size_t)L * D * 4),
               o_n1g = up(w->n1g, (size_t)L * D * 4), o_n1b = up(w->n1b, (size_t)L * D * 4),
               o_n2g = up(w->n2g, (size_t)L * D * 4), o_n2b = up(w->n2b, (size_t)L * D * 4),
               o_pe = up(pe.data(), (size_t)cap * D * 4);
  if (cudaMalloc(&e->wmem, off) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return fail(GSVK_ERR_NOMEM, "t2s_batch_create: weights");
  }
  uint8_t* base = static_cast<uint8_t*>(e->wmem);
  for (const Up& u : ups) {
    int rc = check_cuda(cudaMemcpy(base + u.o, u.src, u.bytes, cudaMemcpyHostToDevice), "upload");
    if (rc) { gsvk_t2s_batch_destroy(e); return rc; }
  }
  d.wqkv = reinterpret_cast<const uint16_t*>(base + o_q);
  d.wout = reinterpret_cast<const uint16_t*>(base + o_o);
  d.w1 = reinterpret_cast<const uint16_t*>(base + o_1);
  d.w2 = reinterpret_cast<const uint16_t*>(base + o_2);
  d.wpred = reinterpret_cast<const uint16_t*>(base + o_p);
  d.emb = reinterpret_cast<const uint16_t*>(base + o_e);
  d.bqkv = reinterpret_cast<const float*>(base + o_bq);
  d.bout = reinterpret_cast<const float*>(base + o_bo);
  d.b1 = reinterpret_cast<const float*>(base + o_b1);
  d.b2 = reinterpret_cast<const float*>(base + o_b2);
  d.n1g = reinterpret_cast<const float*>(base + o_n1g);
  d.n1b = reinterpret_cast<const float*>(base + o_n1b);
  d.n2g = reinterpret_cast<const float*>(base + o_n2g);
  d.n2b = reinterpret_cast<const float*>(base + o_n2b);
  d.pe = reinterpret_cast<const float*>(base + o_pe);
  // KV caches + per-utterance state + activations
  const size_t B = (size_t)max_batch;
  off = 0;
  const size_t o_kc = take(B * L * cap * D * 2), o_vc = take(B * L * cap * D * 2),
               o_bl = take(B * 4), o_bp = take(B * 4), o_st = take(256), o_tok = take(B * 4),
               o_out = take((size_t)max_steps * B * 4), o_mg = take((size_t)max_steps * B * 4),
               o_dn = take(256), o_seen = take(B * V), o_x32 = take(B * D * 4),
               o_qkv = take(B * 3 * D * 4), o_hp = take(B * D * 4), o_h32 = take(B * D * 4),
               o_xp = take(B * D * 4), o_lg = take(B * V * 4), o_x16 = take(B * D * 2),
               o_a16 = take(B * D * 2), o_h16 = take(B * D * 2), o_ff = take(B * F * 2);
  const int max_chunks = (cap + kAttnChunk - 1) / kAttnChunk;
  const size_t o_tk = take(B * 4), o_po = take(B * max_chunks * D * 4),
               o_pm = take(B * max_chunks * H * 8), o_wk = take((size_t)L * 4);
  if (cudaMalloc(&e->amem, off) != cudaSuccess) {
    cudaGetLastError();
    gsvk_t2s_batch_destroy(e);
    return fail(GSVK_ERR_NOMEM, "t2s_batch_create: caches (%zu bytes)", off);
  }
  uint8_t* a = static_cast<uint8_t*>(e->amem);
  if (int rc = check_cuda(cudaMemset(a, 0, off), "t2s_batch memset")) {
    gsvk_t2s_batch_destroy(e);
    return rc;
  }
  d.kc = reinterpret_cast<uint16_t*>(a + o_kc);
  d.vc = reinterpret_cast<uint16_t*>(a + o_vc);
  e->base_len = reinterpret_cast<int32_t*>(a + o_bl);
  e->base_pe = reinterpret_cast<int32_t*>(a + o_bp);
  e->step = reinterpret_cast<int32_t*>(a + o_st);
  e->tok = reinterpret_cast<int32_t*>(a + o_tok);
  e->tokens_out = reinterpret_cast<int32_t*>(a + o_out);
  e->margins = reinterpret_cast<float*>(a + o_mg);
  e->done = reinterpret_cast<unsigned*>(a + o_dn);
  e->seen = a + o_seen;
  e->x32 = reinterpret_cast<float*>(a + o_x32);
  e->qkv32 = reinterpret_cast<float*>(a + o_qkv);
  e->hpre32 = reinterpret_cast<float*>(a + o_hp);
  e->h32 = reinterpret_cast<float*>(a + o_h32);
  e->xpre32 = reinterpret_cast<float*>(a + o_xp);
  e->logits = reinterpret_cast<float*>(a + o_lg);
  e->x16 = reinterpret_cast<uint16_t*>(a + o_x16);
  e->attn16 = reinterpret_cast<uint16_t*>(a + o_a16);
  e->h16 = reinterpret_cast<uint16_t*>(a + o_h16);
  e->ff16 = reinterpret_cast<uint16_t*>(a + o_ff);
  e->ticket = reinterpret_cast<unsigned*>(a + o_tk);
  e->part_o = reinterpret_cast<float*>(a + o_po);
  e->part_ml = reinterpret_cast<float2*>(a + o_pm);
  e->max_chunks = max_chunks;
  e->attn_work = reinterpret_cast<int*>(a + o_wk);
  e->attn_stream = D == 256 || D == 512;
  e->attn_kind = e->attn_stream ? 1 : 0;
  if (e->attn_stream) {
    if (int rc = check_cuda(cudaFuncSetAttribute(D == 512 ? batch_attn_stream_kernel<2>
                                                          : batch_attn_stream_kernel<1>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(attn_stream_smem_bytes(D, H, max_batch))),
                            "streaming attention smem attribute")) {
      gsvk_t2s_batch_destroy(e);
      return rc;
    }
  }
  if (int rc = check_cuda(cudaFuncSetAttribute(batch_attn_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(attn_smem_bytes(D, H))),
                          "attention smem attribute")) {
    gsvk_t2s_batch_destroy(e);
    return rc;
  }
  d.base_len = e->base_len;
  d.base_pe = e->base_pe;
  d.step = e->step;
  d.tok = e->tok;
  d.seen = e->seen;
  d.tokens_out = e->tokens_out;
  d.margins = e->margins;
  *out = e;
  return GSVK_OK;
}

int gsvk_t2s_batch_load_kv(gsvk_t2s_batch_t h, int b, const uint16_t* k_host,
                           const uint16_t* v_host, size_t len, size_t src_rows,
                           gsvk_stream_t stream) {
  if (!h || b < 0 || b >= h->max_batch || (len && (!k_host || !v_host)) || src_rows < len ||
      len > (size_t)h->d.cap)
    return fail(GSVK_ERR_INVALID, "t2s_batch_load_kv: bad arguments");
  const BatchDev& d = h->d;
  for (int l = 0; l < d.L && len; ++l) {
    const size_t dst = (((size_t)b * d.L + l) * d.cap) * d.D;
    int rc = check_cuda(cudaMemcpyAsync(d.kc + dst, k_host + (size_t)l * src_rows * d.D,
                                        len * d.D * 2, cudaMemcpyDefault, as_cuda(stream)),
                        "batch kv k");
    if (rc) return rc;
    rc = check_cuda(cudaMemcpyAsync(d.vc + dst, v_host + (size_t)l * src_rows * d.D, len * d.D * 2,
                                    cudaMemcpyDefault, as_cuda(stream)),
                    "batch kv v");
    if (rc) return rc;
  }
  return GSVK_OK;
}

// Sets the B utterances' lengths, PE origins, first input tokens and
// histories (HOST arrays; hist is [B][n_hist], -1 entries ignored) and
// resets the step counter.
int gsvk_t2s_batch_begin(gsvk_t2s_batch_t h, int B, const int32_t* len, const int32_t* pe0,
                         const int32_t* first_tok, const int32_t* hist, int n_hist,
                         gsvk_stream_t stream) {
  if (!h || B <= 0 || B > h->max_batch || !len || !pe0 || !first_tok || (n_hist > 0 && !hist))
    return fail(GSVK_ERR_INVALID, "t2s_batch_begin: bad arguments");
  const BatchDev& d = h->d;
  for (int b = 0; b < B; ++b)
    if (len[b] < 0 || len[b] + h->max_steps > d.cap || pe0[b] < 0 || pe0[b] + h->max_steps > d.cap ||
        first_tok[b] < 0 || first_tok[b] >= d.V)
      return fail(GSVK_ERR_INVALID, "t2s_batch_begin: utterance %d out of range", b);
  cudaStream_t st = as_cuda(stream);
  std::vector<uint8_t> seen((size_t)B * d.V, 0);
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < n_hist; ++i) {
      const int t = hist[(size_t)b * n_hist + i];
      if (t >= 0 && t < d.V) seen[(size_t)b * d.V + t] = 1;
    }
  // synchronous copies from pageable memory: the caller's arrays may be freed after return
  int rc = check_cuda(cudaMemcpy(h->seen, seen.data(), seen.size(), cudaMemcpyHostToDevice), "seen");
  if (!rc) rc = check_cuda(cudaMemcpy(h->base_len, len, B * 4, cudaMemcpyHostToDevice), "len");
  if (!rc) rc = check_cuda(cudaMemcpy(h->base_pe, pe0, B * 4, cudaMemcpyHostToDevice), "pe0");
  if (!rc) rc = check_cuda(cudaMemcpy(h->tok, first_tok, B * 4, cudaMemcpyHostToDevice), "tok");
  if (!rc) rc = check_cuda(cudaMemsetAsync(h->step, 0, 4, st), "step");
  if (!rc) rc = check_cuda(cudaMemsetAsync(h->done, 0, 4, st), "done");
  h->cur_batch = B;
  h->host_step = 0;
  h->d.B = B;
  return rc;
}

// Runs `steps` greedy steps (no EOS stop: fixed-length batches).  The first
// call for a batch size records the step into a CUDA graph; later steps
// replay it.  Outputs stay on the device until gsvk_t2s_batch_read.
int gsvk_t2s_batch_run(gsvk_t2s_batch_t h, int steps, int use_graph, gsvk_stream_t stream) {
  if (!h || h->cur_batch <= 0 || steps < 0) return fail(GSVK_ERR_INVALID, "t2s_batch_run: begin first");
  if (h->host_step + steps > h->max_steps)
    return fail(GSVK_ERR_INVALID, "t2s_batch_run: %d + %d steps exceed max_steps %d", h->host_step,
                steps, h->max_steps);
  h->host_step += steps;
  cudaStream_t st = as_cuda(stream);
  const int B = h->cur_batch;
  if (!use_graph) {
    for (int s = 0; s < steps; ++s)
      if (int rc = batch_step(h, B, st, &h->launches_per_step)) return rc;
    return GSVK_OK;
  }
  if (!h->exec || h->graph_batch != B) {
    if (h->exec) cudaGraphExecDestroy(h->exec);
    if (h->graph) cudaGraphDestroy(h->graph);
    h->exec = nullptr;
    h->graph = nullptr;
    cudaStream_t cap;
    int rc = check_cuda(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking), "capture stream");
    if (rc) return rc;
    rc = check_cuda(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "begin capture");
    if (!rc) rc = batch_step(h, B, cap, &h->launches_per_step);
    cudaGraph_t g = nullptr;
    const int rc_end = check_cuda(cudaStreamEndCapture(cap, &g), "end capture");
    cudaStreamDestroy(cap);
    if (rc || rc_end) {
      if (g) cudaGraphDestroy(g);
      return rc ? rc : rc_end;
    }
    rc = check_cuda(cudaGraphInstantiate(&h->exec, g, 0), "graph instantiate");
    if (rc) {
      cudaGraphDestroy(g);
      return rc;
    }
    h->graph = g;
    h->graph_batch = B;
  }
  for (int s = 0; s < steps; ++s)
    if (int rc = check_cuda(cudaGraphLaunch(h->exec, st), "graph launch")) return rc;
  return GSVK_OK;
}

// tokens / margins: HOST [steps][B]; synchronous.
int gsvk_t2s_batch_read(gsvk_t2s_batch_t h, int steps, int32_t* tokens, float* margins) {
  if (!h || steps < 0 || steps > h->max_steps || !tokens)
    return fail(GSVK_ERR_INVALID, "t2s_batch_read: bad arguments");
  const size_t n = (size_t)steps * h->cur_batch;
  int rc = check_cuda(cudaMemcpy(tokens, h->tokens_out, n * 4, cudaMemcpyDeviceToHost), "tokens");
  if (!rc && margins)
    rc = check_cuda(cudaMemcpy(margins, h->margins, n * 4, cudaMemcpyDeviceToHost), "margins");
  return rc;
}

// Logits of the last step (HOST [B][V]); synchronous.
int gsvk_t2s_batch_read_logits(gsvk_t2s_batch_t h, float* host_out) {
  if (!h || !host_out) return fail(GSVK_ERR_INVALID, "t2s_batch_read_logits: null");
  return check_cuda(cudaMemcpy(host_out, h->logits, (size_t)h->cur_batch * h->d.V * 4,
                               cudaMemcpyDeviceToHost),
                    "logits");
}

int gsvk_t2s_batch_launches_per_step(gsvk_t2s_batch_t h) { return h ? h->launches_per_step : 0; }

int gsvk_t2s_batch_set_attention(gsvk_t2s_batch_t h, int kind) {
  if (!h) return fail(GSVK_ERR_INVALID, "t2s_batch_set_attention: null handle");
  if (kind < 0 || kind > 1 || (kind == 1 && !h->attn_stream))
    return fail(GSVK_ERR_UNSUPPORTED, "t2s_batch_set_attention: kernel %d not available for this model",
                kind);
  if (kind != h->attn_kind) {  // the captured step holds the previous kernel
    if (h->exec) cudaGraphExecDestroy(h->exec);
    if (h->graph) cudaGraphDestroy(h->graph);
    h->exec = nullptr;
    h->graph = nullptr;
    h->attn_kind = kind;
  }
  return GSVK_OK;
}

int gsvk_t2s_batch_attention(gsvk_t2s_batch_t h) { return h ? h->attn_kind : -1; }

}  // extern "C"
