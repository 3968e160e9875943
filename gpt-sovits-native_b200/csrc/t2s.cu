// t2s.cu — the T2S autoregressive transformer on the device
// (GPT-SoVITS-native src/ar/t2s_engine.cpp), post-LN, fused QKV, ReLU FFN.
//
// All arithmetic follows the canonical association of canon.cuh, which the
// CPU oracle evaluates identically: decode is bit-exact against it.
//
// Prefill (block_prefill_impl, t2s_engine.cpp:881-1034): per layer, four
// canonical-order GEMMs (one warp per 4x4 output tile, fused bias / ReLU /
// residual), a KV append, the chunked-softmax attention and two LayerNorms.
//
// Decode (block_decode_impl + greedy_sample + the generate loop,
// t2s_engine.cpp:1036-1119, 1594-1636, 1839-1900): ONE persistent cooperative
// kernel runs every step of the generation.  Per layer it has five phases
// separated by grid barriers:
//   P1  x = LN2(prev) ; q|k|v = Wqkv . f16(x) + b ; k, v -> fp16 KV slot
//   P2  attention partials per (head, key chunk)  (split-K softmax); the
//       slot that finishes a head's last chunk merges that head's records
//   P3  hpre = Wout . f16(attn) + b + x
//   P4  h = LN1(hpre) ; ff = relu(W1 . f16(h) + b)
//   P5  xpre = W2 . ff + b + h          (fp32 activations, as the reference)
// then logits = Wpred . LN2(xpre) and every CTA redundantly applies the
// repetition penalty and takes the argmax, so the next token's embedding
// needs no extra barrier.  Each CTA owns fixed row slices of every weight
// matrix and streams them into shared memory one layer ahead with bulk
// copies, so HBM streaming overlaps the barrier latency chain.
#include <chrono>
#include <cmath>
#include <mutex>
#include <cstring>
#include <vector>

#include "canon.cuh"
#include "gsvk_internal.hpp"

struct gsvk_t2s;

namespace gsvk {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 64;       // softmax chunk (slots), fixed by the canonical order
constexpr int kMaxChunks = 256;  // chunks per head (cap <= 16384 slots)
constexpr int kSlots = kThreads / 64;  // concurrent attention chunks per CTA
constexpr uint32_t kGridSpin = 1u << 23;

struct T2SDev {
  int L, D, H, F, V, cap, HD;
  float eps, alpha, scale;
  const uint16_t *wqkv, *wout, *w1, *w2, *wpred, *emb;
  const uint16_t* w2p;  // W2 rows in the lane order of t2s_cluster_kernel (or null)
  const float *bqkv, *bout, *b1, *b2, *n1g, *n1b, *n2g, *n2b, *pe;
  uint16_t *kc, *vc;
  float *q, *part, *hpre, *ff, *xpre, *logits;
  float* attn;       // [D] merged attention output (fp16-rounded), written by each head's merger
  unsigned* ticket;  // [H] chunk records finished per head (zero between layers)
  unsigned* bar;
  uint32_t* status;
};

struct DecodeArgs {
  int pos0;       // KV slot of the first decoded token
  int pe0;        // position-encoding index of the first decoded token (= P)
  int max_steps;
  int stop_on_eos;
  const int32_t* hist;
  int n_hist;
  int32_t* tokens;
  int* n_out;
  float* margins;
  // shared-memory plan (identical in every CTA)
  int mq, mo, m1, m2, ml;  // max rows per CTA of qkv / out / w1 / w2 / logits
  uint32_t layer_bytes;
  uint32_t ln_off;   // LayerNorm parameters inside a layer buffer: n1g, n1b of the
                     // layer, then n2g, n2b of the layer before it (fp32, D each)
  // sampling (SamplingParams, t2s_engine.hpp:69-77): mode 0 greedy, 1 top-k
  int samp_mode, samp_top_k;
  float samp_top_p, samp_temp, samp_pen;
  unsigned long long samp_seed;
  // optional phase trace: CTA 0 writes %globaltimer (ns) at every phase
  // boundary of the first kTraceSteps steps, kTraceStride slots per step
  unsigned long long* trace;
};

constexpr int kTraceSteps = 4;
constexpr int kTraceStride = 16 + 16 * 64;

__host__ __device__ inline int row_lo(int rows, int g, int c) {
  return static_cast<int>(static_cast<long long>(rows) * c / g);
}

// ----------------------------------------------------------- block helpers
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier on a monotonically increasing counter (reset by the host
// before each launch).  Bounded: on timeout, or when another CTA has already
// flagged one, it returns false and the kernel winds down.
// `during` runs on every other thread while thread 0 waits (work that needs
// the CTA barrier but not the grid one, e.g. issuing the next prefetch).
template <typename During>
__device__ bool grid_sync_and(unsigned* bar, unsigned& epoch, uint32_t* status, int* flag,
                              During&& during) {
  __syncthreads();
  if (threadIdx.x == 0) {
    ++epoch;
    const unsigned target = epoch * gridDim.x;
    // one release-add publishes this CTA's writes (made visible to thread 0
    // by the CTA barrier above) and arrives
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    int ok = 1;
    for (uint32_t i = 0;; ++i) {
      const unsigned v = ld_acquire(bar);
      if (static_cast<int>(v - target) >= 0) break;
      if ((i & 1023u) == 1023u && *reinterpret_cast<volatile uint32_t*>(status) != 0) {
        ok = 0;
        break;
      }
      if (i > kGridSpin) {
        atomicExch(status, DEV_TIMEOUT);
        ok = 0;
        break;
      }
    }
    *flag = ok;  // the acquire load above orders everything after it
  } else {
    during();
  }
  __syncthreads();
  return *flag != 0;
}
__device__ bool grid_sync(unsigned* bar, unsigned& epoch, uint32_t* status, int* flag) {
  return grid_sync_and(bar, epoch, status, flag, [] {});
}

__device__ __forceinline__ void slot_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

// Floats of shared memory one attention slot uses: q[64], e[64], red[8],
// staged V rows (64 x HD halves).
template <int HD>
__host__ __device__ constexpr int slot_floats() {
  return 64 + 64 + 8 + kChunk * HD / 2;
}

// One 64-slot chunk [k0, k1) of the canonical softmax for one head, by a
// slot of 64 threads (two warps, named barrier `bar_id`): thread t scores key
// k0 + t with the dot_f16kv order (its K row read straight into registers),
// stages its V row, then the slot forms the chunk max, exp_det weights and the
// two sequential sums (l, and o one dimension per lane).  dst <- {m, l, o[HD]}.
template <int HD>
__device__ void attn_chunk_slot(const float* qg, bool q_global, const uint16_t* kcache,
                                const uint16_t* vcache, int D, int k0, int k1, float scale,
                                float* sm, int bar_id, float* dst) {
  float* ew = sm + 64;
  float* red = sm + 128;
  uint16_t* vst = reinterpret_cast<uint16_t*>(sm + 136);
  const int t = threadIdx.x & 63, lane = t & 31, w = t >> 5;
  const int nk = k1 - k0;
  constexpr int kV = HD / 8;
  // every global load of the chunk in flight at once: q (broadcast), K row, V row
  float q[HD];
  uint4 kr[kV], vr[kV];
  const int kk = t < nk ? t : 0;
  const uint4* ks = reinterpret_cast<const uint4*>(kcache + static_cast<size_t>(k0 + kk) * D);
  const uint4* vs = reinterpret_cast<const uint4*>(vcache + static_cast<size_t>(k0 + kk) * D);
#pragma unroll
  for (int p = 0; p < HD / 4; ++p) {
    const float4 v = q_global ? __ldcg(reinterpret_cast<const float4*>(qg) + p)
                              : reinterpret_cast<const float4*>(qg)[p];
    q[4 * p] = v.x;
    q[4 * p + 1] = v.y;
    q[4 * p + 2] = v.z;
    q[4 * p + 3] = v.w;
  }
#pragma unroll
  for (int p = 0; p < kV; ++p) {
    kr[p] = __ldcg(ks + p);
    vr[p] = __ldcg(vs + p);
  }
#pragma unroll
  for (int p = 0; p < kV; ++p) reinterpret_cast<uint4*>(vst + t * HD)[p] = vr[p];
  float score = -INFINITY;
  if (t < nk) score = __fmul_rn(thread_dot_kv<HD>(q, kr), scale);
  float mx = warp_max(score);
  if (lane == 0) red[w] = mx;
  slot_sync(bar_id);
  mx = fmaxf(red[0], red[1]);
  ew[t] = t < nk ? exp_det(__fsub_rn(score, mx)) : 0.f;
  slot_sync(bar_id);
  // o: dimension d = 32*w + lane (HD = 64) or lane (HD = 32, warp 0);
  // l: warp 1 lane 0.
  float o = 0.f, l = 0.f;
  const bool do_o = (HD == 64) || (w == 0);
  const bool do_l = (w == 1 && lane == 0);
  const int d = (HD == 64 ? 32 * w : 0) + lane;
  int k = 0;
  for (; k + 8 <= nk; k += 8) {
    float e8[8], v8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      e8[u] = ew[k + u];
      v8[u] = do_o ? h2f(vst[(k + u) * HD + d]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (do_o) o = __fadd_rn(o, __fmul_rn(e8[u], v8[u]));
      if (do_l) l = __fadd_rn(l, e8[u]);
    }
  }
  for (; k < nk; ++k) {
    const float e = ew[k];
    if (do_o) o = __fadd_rn(o, __fmul_rn(e, h2f(vst[k * HD + d])));
    if (do_l) l = __fadd_rn(l, e);
  }
  if (do_o) dst[4 + d] = o;
  if (do_l) {
    dst[0] = mx;
    dst[1] = l;
  }
  slot_sync(bar_id);
}

// Chunk records are {m, l, pad, pad, o[HD]}: HD + 4 floats, 16-byte aligned.
template <int HD>
__host__ __device__ constexpr int rec_floats() {
  return HD + 4;
}

// Combine nch chunk records of one head; one warp, every lane returns dims
// lane (and lane+32).
template <int HD>
__device__ __forceinline__ void attn_combine(const float* rec, int nch, bool cg, float* out0,
                                             float* out1) {
  const int lane = threadIdx.x & 31;
  auto rd = [cg](const float* p) { return cg ? __ldcg(p) : *p; };
  float M = -INFINITY;
  for (int c = 0; c < nch; ++c) M = fmaxf(M, rd(rec + c * rec_floats<HD>()));
  float L = 0.f, O0 = 0.f, O1 = 0.f;
  for (int c = 0; c < nch; ++c) {
    const float* r = rec + c * rec_floats<HD>();
    const float w = exp_det(__fsub_rn(rd(r), M));
    L = __fadd_rn(L, __fmul_rn(rd(r + 1), w));
    O0 = __fadd_rn(O0, __fmul_rn(rd(r + 4 + lane), w));
    if (HD > 32) O1 = __fadd_rn(O1, __fmul_rn(rd(r + 4 + 32 + lane), w));
  }
  const float inv = __fdiv_rn(1.0f, L);
  *out0 = __fmul_rn(O0, inv);
  *out1 = HD > 32 ? __fmul_rn(O1, inv) : 0.f;
}

// dst[0, n) <- src (global, written by other CTAs), n a multiple of 4: every
// thread issues all of its float4 loads before the first store.
template <int MAXV>
__device__ __forceinline__ void load_vec(float* dst, const float* src, int n) {
  const int nv = n >> 2;
  float4 r[MAXV];
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int i = threadIdx.x + u * kThreads;
    if (i < nv) r[u] = __ldcg(reinterpret_cast<const float4*>(src) + i);
  }
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int i = threadIdx.x + u * kThreads;
    if (i < nv) reinterpret_cast<float4*>(dst)[i] = r[u];
  }
  for (int i = threadIdx.x + MAXV * kThreads; i < nv; i += kThreads)
    reinterpret_cast<float4*>(dst)[i] = __ldcg(reinterpret_cast<const float4*>(src) + i);
}

struct Slices {
  int q0, q1, o0, o1, a0, a1, b0, b1, l0, l1;
};

__device__ Slices my_slices(const T2SDev& m) {
  const int G = gridDim.x, c = blockIdx.x;
  Slices s;
  s.q0 = row_lo(3 * m.D, G, c);
  s.q1 = row_lo(3 * m.D, G, c + 1);
  s.o0 = row_lo(m.D, G, c);
  s.o1 = row_lo(m.D, G, c + 1);
  s.a0 = row_lo(m.F, G, c);
  s.a1 = row_lo(m.F, G, c + 1);
  s.b0 = row_lo(m.D, G, c);
  s.b1 = row_lo(m.D, G, c + 1);
  s.l0 = row_lo(m.V, G, c);
  s.l1 = row_lo(m.V, G, c + 1);
  return s;
}

// Part `part` (0..4) of streaming this CTA's slices of layer l into `buf`:
// 0 posts the byte count of the whole layer (one arrival) and copies the QKV
// slice, 1 the out slice, 2 the W1 slice, 3 the W2 slice, 4 the LayerNorm
// vectors (every CTA normalises full rows: n1 of layer l, n2 of layer l - 1).
// The parts may be issued by different threads, in any order (the copies'
// bytes may land before the count is posted: the phase cannot complete
// before the arrival).
__device__ void prefetch_part(const T2SDev& m, const DecodeArgs& a, const Slices& s, int l,
                              uint8_t* buf, uint64_t* bar, int part) {
  const size_t D = m.D, F = m.F;
  const uint32_t bq = (s.q1 - s.q0) * D * 2, bo = (s.o1 - s.o0) * D * 2,
                 b1 = (s.a1 - s.a0) * D * 2, b2 = (s.b1 - s.b0) * F * 2;
  const uint32_t vb = static_cast<uint32_t>(D) * 4;
  uint8_t* pq = buf;
  uint8_t* po = pq + static_cast<size_t>(a.mq) * D * 2;
  uint8_t* p1 = po + static_cast<size_t>(a.mo) * D * 2;
  uint8_t* p2 = p1 + static_cast<size_t>(a.m1) * D * 2;
  switch (part) {
    case 0:
      mbar_arrive_expect_tx(bar, bq + bo + b1 + b2 + (l > 0 ? 4 * vb : 2 * vb));
      if (bq) bulk_load(pq, m.wqkv + (static_cast<size_t>(l) * 3 * D + s.q0) * D, bq, bar);
      break;
    case 1:
      if (bo) bulk_load(po, m.wout + (static_cast<size_t>(l) * D + s.o0) * D, bo, bar);
      break;
    case 2:
      if (b1) bulk_load(p1, m.w1 + (static_cast<size_t>(l) * F + s.a0) * D, b1, bar);
      break;
    case 3: {
      const uint16_t* w2 = m.w2p ? m.w2p : m.w2;  // the lane-ordered copy when there is one
      if (b2) bulk_load(p2, w2 + (static_cast<size_t>(l) * D + s.b0) * F, b2, bar);
      break;
    }
    default: {
      float* ln = reinterpret_cast<float*>(buf + a.ln_off);
      bulk_load(ln, m.n1g + static_cast<size_t>(l) * D, vb, bar);
      bulk_load(ln + D, m.n1b + static_cast<size_t>(l) * D, vb, bar);
      if (l > 0) {
        bulk_load(ln + 2 * D, m.n2g + static_cast<size_t>(l - 1) * D, vb, bar);
        bulk_load(ln + 3 * D, m.n2b + static_cast<size_t>(l - 1) * D, vb, bar);
      }
    }
  }
}
// One thread: the whole layer.
__device__ void prefetch_layer(const T2SDev& m, const DecodeArgs& a, const Slices& s, int l,
                               uint8_t* buf, uint64_t* bar) {
  for (int part = 0; part < 5; ++part) prefetch_part(m, a, s, l, buf, bar, part);
}

#include "t2s_cluster.cuh"
#include "t2s_flow.cuh"

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) t2s_decode_kernel(const T2SDev m, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<128>(smem_raw);
  const int D = m.D, F = m.F, V = m.V, H = m.H, L = m.L;
  uint8_t* wbuf[2] = {smem, smem + a.layer_bytes};
  uint16_t* wlog = reinterpret_cast<uint16_t*>(smem + 2 * static_cast<size_t>(a.layer_bytes));
  float* lnf = reinterpret_cast<float*>(wlog + static_cast<size_t>(a.ml) * D);  // last LN2 g, b
  float* slots = lnf + 2 * D;                                                  // attention
  float* xs = slots + kSlots * slot_floats<HD>();         // layer input x
  float* hs = xs + D;                                     // LN1 output h
  float* act = hs + D;                                    // operand, max(D, F)
  float* sc = act + (F > D ? F : D);                      // chunk scores / weights
  float* red = sc + kChunk;                               // 64 floats
  int* flag = reinterpret_cast<int*>(red + 64);
  int* tokp = flag + 4;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(tokp + 4);
  float* bsm = reinterpret_cast<float*>(mbar + 4);  // this layer's bias slices
  uint8_t* seen = reinterpret_cast<uint8_t*>(bsm + ((a.mq + a.mo + a.m1 + a.m2 + 3) & ~3));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const Slices s = my_slices(m);
  const int nq = s.q1 - s.q0, no = s.o1 - s.o0, na = s.a1 - s.a0, nb = s.b1 - s.b0;
  // bias element `tid` of layer l's row slices (QKV, out, W1, W2 in order)
  auto bias_of = [&](int l) -> float {
    const size_t L_ = static_cast<size_t>(l);
    if (tid < nq) return __ldg(m.bqkv + L_ * 3 * D + s.q0 + tid);
    if (tid < nq + no) return __ldg(m.bout + L_ * D + s.o0 + tid - nq);
    if (tid < nq + no + na) return __ldg(m.b1 + L_ * F + s.a0 + tid - nq - no);
    if (tid < nq + no + na + nb) return __ldg(m.b2 + L_ * D + s.b0 + tid - nq - no - na);
    return 0.f;
  };
  float bias_next = 0.f;
  unsigned epoch = 0;
  uint32_t uses[2] = {0, 0};
  const int eos = V - 1;

  for (int c = tid; c < V; c += kThreads) seen[c] = 0;
  __syncthreads();
  for (int i = tid; i < a.n_hist; i += kThreads) {
    const int t = a.hist[i];
    if (t >= 0 && t < V) seen[t] = 1;
  }
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    mbar_init(&mbar[2], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bl = (s.l1 - s.l0) * D * 2;
    mbar_arrive_expect_tx(&mbar[2], bl + 2u * D * 4);
    if (bl) bulk_load(wlog, m.wpred + static_cast<size_t>(s.l0) * D, bl, &mbar[2]);
    bulk_load(lnf, m.n2g + static_cast<size_t>(L - 1) * D, D * 4, &mbar[2]);
    bulk_load(lnf + D, m.n2b + static_cast<size_t>(L - 1) * D, D * 4, &mbar[2]);
    // the global layer sequence g = 0, 1, 2, ... runs layer g % L from buffer g & 1
    prefetch_layer(m, a, s, 0, wbuf[0], &mbar[0]);
    prefetch_layer(m, a, s, 1 % L, wbuf[1], &mbar[1]);
  }
  uint32_t pending[2] = {1u, 1u};
  unsigned gl = 0;
  bool alive = mbar_wait(&mbar[2], 0, m.status);

  int n_out = 0;
  unsigned long long* tr = nullptr;
#define GSVK_TR(slot)                                   \
  do {                                                  \
    if (tr && tid == 0) tr[(slot)] = global_ns();       \
  } while (0)
  for (int idx = 0; idx < a.max_steps && alive; ++idx) {
    tr = (a.trace && blockIdx.x == 0 && idx < kTraceSteps) ? a.trace + idx * kTraceStride : nullptr;
    GSVK_TR(0);
    bias_next = bias_of(0);  // in flight during the sampling
    // ------------------------------------------------ greedy sample (all CTAs)
    // t2s_engine.cpp:1594-1636: penalty once per distinct history token,
    // EOS excluded while idx < 11, first maximum wins.
    const int eos_allowed = idx >= 11;
    const int limit = eos_allowed ? V : V - 1;
    float bv = -INFINITY, sv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = tid; c < limit; c += kThreads) {
      float v = __ldcg(m.logits + c);
      if (seen[c]) v = v < 0.f ? __fmul_rn(v, 1.35f) : __fdiv_rn(v, 1.35f);
      if (v > bv || (v == bv && c < bi)) {
        sv = bv;
        bv = v;
        bi = c;
      } else if (v > sv) {
        sv = v;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const float os = __shfl_xor_sync(0xffffffffu, sv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        sv = fmaxf(os, bv);
        bv = ov;
        bi = oi;
      } else {
        sv = fmaxf(sv, ov);
      }
    }
    __syncthreads();
    if (lane == 0) {
      red[warp] = bv;
      red[kWarps + warp] = sv;
      reinterpret_cast<int*>(red + 2 * kWarps)[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float B = red[0], S = red[kWarps];
      int I = reinterpret_cast<int*>(red + 2 * kWarps)[0];
      for (int w = 1; w < kWarps; ++w) {
        const float ov = red[w], os = red[kWarps + w];
        const int oi = reinterpret_cast<int*>(red + 2 * kWarps)[w];
        if (ov > B || (ov == B && oi < I)) {
          S = fmaxf(os, B);
          B = ov;
          I = oi;
        } else {
          S = fmaxf(S, ov);
        }
      }
      tokp[0] = I;
      if (blockIdx.x == 0 && a.margins) a.margins[idx] = __fsub_rn(B, S);
    }
    __syncthreads();
    const int tok = tokp[0];
    bool stop = false;
    if (a.stop_on_eos && eos_allowed && tok == eos) {
      stop = true;
    } else {
      if (blockIdx.x == 0 && tid == 0) a.tokens[n_out] = tok;
      ++n_out;
      if (tid == 0) seen[tok] = 1;
    }
    if (idx + 1 == a.max_steps) stop = true;
    __syncthreads();
    GSVK_TR(1);
    if (stop) break;

    // ------------------------------------- next input: emb[tok] + alpha*PE
    const int pos = a.pos0 + idx;
    const int len = pos + 1;
    {
      const uint16_t* er = m.emb + static_cast<size_t>(tok) * D;
      const float* pr = m.pe + static_cast<size_t>(a.pe0 + idx) * D;
      for (int i = tid; i < D; i += kThreads) xs[i] = fmaf(m.alpha, pr[i], h2f(er[i]));
    }
    __syncthreads();
    const int nch = (len + kChunk - 1) / kChunk;

    for (int l = 0; l < L && alive; ++l, ++gl) {
      const int b = static_cast<int>(gl & 1u);
      const uint16_t* Wq = reinterpret_cast<const uint16_t*>(wbuf[b]);
      const uint16_t* Wo = Wq + static_cast<size_t>(a.mq) * D;
      const uint16_t* W1 = Wo + static_cast<size_t>(a.mo) * D;
      const uint16_t* W2 = W1 + static_cast<size_t>(a.m1) * D;
      // ---------------------------------------------------------------- P1
      // this layer's buffer: weight slices and the LayerNorm vectors
      if (!mbar_wait(&mbar[b], uses[b] & 1u, m.status)) {
        alive = false;
        break;
      }
      ++uses[b];
      pending[b] = 0;
      const float* lnb = reinterpret_cast<const float*>(wbuf[b] + a.ln_off);
      GSVK_TR(16 + 16 * l + 11);
      if (tid < nq + no + na + nb) bsm[tid] = bias_next;  // loaded a phase ago
      {  // warm L2 with the K / V rows this thread reads in P2 (all but the new key)
        const uint16_t* kc_l = m.kc + static_cast<size_t>(l) * m.cap * D;
        const uint16_t* vc_l = m.vc + static_cast<size_t>(l) * m.cap * D;
        for (int it = blockIdx.x * kSlots + (tid >> 6); it < H * nch; it += G * kSlots) {
          const int h = it / nch, k = (it - h * nch) * kChunk + (tid & 63);
          if (k < len - 1) {
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kc_l + static_cast<size_t>(k) * D + h * HD));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(vc_l + static_cast<size_t>(k) * D + h * HD));
          }
        }
      }
      if (l > 0) {
        load_vec<2>(xs, m.xpre, D);
        __syncthreads();
        GSVK_TR(16 + 16 * l + 14);
        ln_canon(xs, lnb + 2 * D, lnb + 3 * D, D, m.eps, red, act);  // LN2 of layer l - 1
        GSVK_TR(16 + 16 * l + 15);
      } else {
        for (int i = tid; i < D; i += kThreads) act[i] = h2f(f2h(xs[i]));
        __syncthreads();
      }
      GSVK_TR(16 + 16 * l + 10);
      {
        uint16_t* kl = m.kc + (static_cast<size_t>(l) * m.cap + pos) * D;
        uint16_t* vl = m.vc + (static_cast<size_t>(l) * m.cap + pos) * D;
        auto put = [&](int r, float acc) {
          const float v = __fadd_rn(acc, bsm[r - s.q0]);
          if (r < D)
            m.q[r] = v;
          else if (r < 2 * D)
            kl[r - D] = f2h(v);
          else
            vl[r - 2 * D] = f2h(v);
        };
        for (int r = s.q0 + 2 * warp; r < s.q1; r += 2 * kWarps) {
          if (r + 1 < s.q1) {
            float a0, a1;
            warp_dot32x2(Wq + static_cast<size_t>(r - s.q0) * D,
                         Wq + static_cast<size_t>(r + 1 - s.q0) * D, act, D, &a0, &a1);
            if (lane == 0) {
              put(r, a0);
              put(r + 1, a1);
            }
          } else {
            const float a0 = warp_dot32(Wq + static_cast<size_t>(r - s.q0) * D, act, D);
            if (lane == 0) put(r, a0);
          }
        }
      }
      GSVK_TR(16 + 16 * l + 0);
      if (!grid_sync(m.bar, epoch, m.status, flag)) { alive = false; break; }
      GSVK_TR(16 + 16 * l + 1);
      // ---------------------------------------------------------------- P2
      if (l + 1 < L) bias_next = bias_of(l + 1);  // the next layer's, a phase ahead
      {
        const int slot = tid >> 6;
        float* sm = slots + slot * slot_floats<HD>();
        for (int base = blockIdx.x * kSlots; base < H * nch; base += G * kSlots) {
          const int item = base + slot;
          if (item >= H * nch) break;
          const int h = item / nch, c = item - (item / nch) * nch;
          const int k0 = c * kChunk, k1 = min(len, k0 + kChunk);
          attn_chunk_slot<HD>(m.q + h * HD, true, m.kc + static_cast<size_t>(l) * m.cap * D + h * HD,
                              m.vc + static_cast<size_t>(l) * m.cap * D + h * HD, D, k0, k1, m.scale,
                              sm, 1 + slot,
                              m.part + (static_cast<size_t>(h) * kMaxChunks + c) * rec_floats<HD>());
          // The slot that finishes the last record of head h merges the
          // head's records (canonical chunk order) right away.  One
          // acq_rel ticket per record: its release publishes the record the
          // slot just wrote (ordered before it by the slot barrier inside
          // attn_chunk_slot); its acquire, for the last ticket, makes every
          // other record visible to this slot.
          int* last = reinterpret_cast<int*>(sm + 128 + 4);
          if ((tid & 63) == 0) {
            unsigned old;
            asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                         : "=r"(old)
                         : "l"(m.ticket + h)
                         : "memory");
            *last = old == static_cast<unsigned>(nch - 1);
          }
          slot_sync(1 + slot);
          if (*last) {
            const float* rec = m.part + static_cast<size_t>(h) * kMaxChunks * rec_floats<HD>();
            const int n4 = nch * rec_floats<HD>() / 4;
            // staged into the slot's V area (sm + 136), clear of the flag at sm[132]
            float* stg = sm + 136;
            const bool fits = n4 * 4 <= kChunk * HD / 2;
            if (fits) {  // stage the records, every load in flight
              constexpr int kPer = 4;
              float4 r[kPer];
              const int t64 = tid & 63;
#pragma unroll
              for (int u = 0; u < kPer; ++u)
                if (t64 + 64 * u < n4) r[u] = __ldcg(reinterpret_cast<const float4*>(rec) + t64 + 64 * u);
#pragma unroll
              for (int u = 0; u < kPer; ++u)
                if (t64 + 64 * u < n4) reinterpret_cast<float4*>(stg)[t64 + 64 * u] = r[u];
              for (int i = t64 + 64 * kPer; i < n4; i += 64)
                reinterpret_cast<float4*>(stg)[i] = __ldcg(reinterpret_cast<const float4*>(rec) + i);
            }
            slot_sync(1 + slot);
            if ((tid & 63) < 32) {
              float o0, o1;
              attn_combine<HD>(fits ? stg : rec, nch, !fits, &o0, &o1);
              m.attn[h * HD + lane] = h2f(f2h(o0));
              if (HD > 32) m.attn[h * HD + 32 + lane] = h2f(f2h(o1));
              if (lane == 0) m.ticket[h] = 0;
            }
          }
          slot_sync(1 + slot);
        }
      }
      GSVK_TR(16 + 16 * l + 2);
      if (!grid_sync(m.bar, epoch, m.status, flag)) { alive = false; break; }
      GSVK_TR(16 + 16 * l + 3);
      // ---------------------------------------------------------------- P3
      load_vec<2>(act, m.attn, D);
      __syncthreads();
      {
        for (int r = s.o0 + warp; r < s.o1; r += kWarps) {
          const float acc = warp_dot32(Wo + static_cast<size_t>(r - s.o0) * D, act, D);
          if (lane == 0) m.hpre[r] = __fadd_rn(__fadd_rn(acc, bsm[nq + r - s.o0]), xs[r]);
        }
      }
      GSVK_TR(16 + 16 * l + 4);
      if (!grid_sync(m.bar, epoch, m.status, flag)) { alive = false; break; }
      GSVK_TR(16 + 16 * l + 5);
      // ---------------------------------------------------------------- P4
      load_vec<2>(hs, m.hpre, D);
      __syncthreads();
      ln_canon(hs, lnb, lnb + D, D, m.eps, red, act);
      GSVK_TR(16 + 16 * l + 12);
      {
        auto put = [&](int r, float acc) {
          const float v = __fadd_rn(acc, bsm[nq + no + r - s.a0]);
          m.ff[r] = v > 0.f ? v : 0.f;
        };
        for (int r = s.a0 + 2 * warp; r < s.a1; r += 2 * kWarps) {
          if (r + 1 < s.a1) {
            float a0, a1;
            warp_dot32x2(W1 + static_cast<size_t>(r - s.a0) * D,
                         W1 + static_cast<size_t>(r + 1 - s.a0) * D, act, D, &a0, &a1);
            if (lane == 0) {
              put(r, a0);
              put(r + 1, a1);
            }
          } else {
            const float a0 = warp_dot32(W1 + static_cast<size_t>(r - s.a0) * D, act, D);
            if (lane == 0) put(r, a0);
          }
        }
      }
      GSVK_TR(16 + 16 * l + 6);
      if (!grid_sync(m.bar, epoch, m.status, flag)) { alive = false; break; }
      GSVK_TR(16 + 16 * l + 7);
      // ---------------------------------------------------------------- P5
      load_vec<4>(act, m.ff, F);
      __syncthreads();
      GSVK_TR(16 + 16 * l + 13);
      if (m.w2p) {  // lane-ordered W2 slice (F = kClF), activations in registers
        float xr[2 * kClFB];
        lane_load_x(act, xr);
        for (int r = s.b0 + warp; r < s.b1; r += kWarps) {
          const float acc = lane_dot_ordered(W2 + static_cast<size_t>(r - s.b0) * F, xr);
          if (lane == 0) m.xpre[r] = __fadd_rn(__fadd_rn(acc, bsm[nq + no + na + r - s.b0]), hs[r]);
        }
      } else {
        for (int r = s.b0 + warp; r < s.b1; r += kWarps) {
          const float acc = warp_dot32(W2 + static_cast<size_t>(r - s.b0) * F, act, F);
          if (lane == 0) m.xpre[r] = __fadd_rn(__fadd_rn(acc, bsm[nq + no + na + r - s.b0]), hs[r]);
        }
      }
      pending[b] = 1;
      GSVK_TR(16 + 16 * l + 8);
      // after the CTA barrier every warp is done with wbuf[b]: it is refilled
      // with global layer gl + 2 while thread 0 waits at the grid barrier
      if (!grid_sync_and(m.bar, epoch, m.status, flag, [&] {
            // the five parts issued in parallel by lane 0 of warps 1..5
            if (lane == 0 && warp >= 1 && warp <= 5)
              prefetch_part(m, a, s, (l + 2) % L, wbuf[b], &mbar[b], warp - 1);
          })) {
        alive = false;
        break;
      }
      GSVK_TR(16 + 16 * l + 9);
    }
    if (!alive) break;
    // ---------------------------------------------------------------- logits
    load_vec<2>(xs, m.xpre, D);
    __syncthreads();
    ln_canon(xs, lnf, lnf + D, D,
             m.eps, red);
    for (int r = s.l0 + warp; r < s.l1; r += kWarps) {
      const float acc = warp_dot32(wlog + static_cast<size_t>(r - s.l0) * D, xs, D);
      if (lane == 0) m.logits[r] = acc;
    }
    GSVK_TR(2);
    if (!grid_sync(m.bar, epoch, m.status, flag)) { alive = false; break; }
    GSVK_TR(3);
  }
#undef GSVK_TR
  // Drain bulk copies still in flight before the CTA exits.
  if (tid == 0) {
    for (int b = 0; b < 2; ++b)
      if (pending[b]) mbar_wait(&mbar[b], uses[b] & 1u, m.status);
    if (blockIdx.x == 0 && a.n_out) *a.n_out = n_out;
  }
  __syncthreads();
}

// ------------------------------------------------------------ prefill kernels
__global__ void embed_kernel(const int32_t* __restrict__ ids, int P, const uint16_t* __restrict__ emb,
                             const float* __restrict__ pe, int pe0, float alpha, int D,
                             float* __restrict__ x, uint16_t* __restrict__ x16) {
  const int t = blockIdx.x;
  const uint16_t* er = emb + static_cast<size_t>(ids[t]) * D;
  const float* pr = pe + static_cast<size_t>(pe0 + t) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = fmaf(alpha, pr[i], h2f(er[i]));
    x[static_cast<size_t>(t) * D + i] = v;
    x16[static_cast<size_t>(t) * D + i] = f2h(v);
  }
}

__global__ void kv_append_kernel(const float* __restrict__ qkv, int S, int D, uint16_t* kc,
                                 uint16_t* vc, int pos) {
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    kc[static_cast<size_t>(pos + t) * D + i] = f2h(qkv[static_cast<size_t>(t) * 3 * D + D + i]);
    vc[static_cast<size_t>(pos + t) * D + i] = f2h(qkv[static_cast<size_t>(t) * 3 * D + 2 * D + i]);
  }
}

// C[m, n] = epi(dot32(B[n], A[m])), A and B fp16 row-major; one warp per 4x4
// output tile, each output's 32 canonical accumulators spread over the lanes.
// epi: + bias[n], ReLU, + residual[m, n], stored as fp32 and/or fp16.
__global__ void __launch_bounds__(256) canon_gemm_kernel(
    const uint16_t* __restrict__ A, int lda, const uint16_t* __restrict__ B, int ldb, int M, int N,
    int K, const float* __restrict__ bias, int relu, const float* __restrict__ res, int ldr,
    float* __restrict__ c32, int ldc, uint16_t* __restrict__ c16, int ldc16) {
  const int lane = threadIdx.x & 31;
  const long long wid = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
  const int n_tiles = (N + 3) / 4;
  const long long mt = wid / n_tiles;
  const int nt = static_cast<int>(wid - mt * n_tiles);
  if (mt * 4 >= M) return;
  int mr[4], nr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mr[i] = min(static_cast<int>(mt * 4) + i, M - 1);
    nr[i] = min(nt * 4 + i, N - 1);
  }
  const int o0 = 8 * (lane >> 2) + (lane & 3);
  const int vec_end = K & ~63;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k = 0; k < vec_end; k += 64) {
    float alo[4], ahi[4], blo[4], bhi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t* ar = A + static_cast<size_t>(mr[i]) * lda + k + o0;
      alo[i] = h2f(ar[0]);
      ahi[i] = h2f(ar[4]);
      const uint16_t* br = B + static_cast<size_t>(nr[i]) * ldb + k + o0;
      blo[i] = h2f(br[0]);
      bhi[i] = h2f(br[4]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = fmaf(blo[j], alo[i], acc[i][j]);
        acc[i][j] = fmaf(bhi[j], ahi[i], acc[i][j]);
      }
  }
  float outv = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = acc[i][j];
      const float t = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
      const float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
      float sum = __shfl_sync(0xffffffffu, u, 0);
#pragma unroll
      for (int g = 1; g < 8; ++g) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, u, 4 * g));
      for (int k = vec_end; k < K; ++k)
        sum = fmaf(h2f(B[static_cast<size_t>(nr[j]) * ldb + k]), h2f(A[static_cast<size_t>(mr[i]) * lda + k]), sum);
      if (lane == i * 4 + j) outv = sum;
    }
  if (lane < 16) {
    const int i = lane >> 2, j = lane & 3;
    const int mm = static_cast<int>(mt * 4) + i, nn = nt * 4 + j;
    if (mm < M && nn < N) {
      float v = outv;
      if (bias) v = __fadd_rn(v, bias[nn]);
      if (relu) v = v > 0.f ? v : 0.f;
      if (res) v = __fadd_rn(v, res[static_cast<size_t>(mm) * ldr + nn]);
      if (c32) c32[static_cast<size_t>(mm) * ldc + nn] = v;
      if (c16) c16[static_cast<size_t>(mm) * ldc16 + nn] = f2h(v);
    }
  }
}

// y[r] = dot32(W[r], x) with fp32 x (logits head), one warp per row.
__global__ void canon_gemv_kernel(const uint16_t* __restrict__ w, const float* __restrict__ x,
                                  float* __restrict__ y, int out, int in) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= out) return;
  const float acc = warp_dot32(w + static_cast<size_t>(r) * in, x, in);
  if ((threadIdx.x & 31) == 0) y[r] = acc;
}

// Masked prefill attention (t2s_engine.cpp:944-979) in the canonical chunked
// softmax: query q of the block sees slots [0, pos + max(text_len, q+1)).
// One CTA per (query, head); its four 64-thread slots take the chunks in
// turn, then warp 0 combines the chunk records in order.
template <int HD>
__global__ void __launch_bounds__(kThreads) prefill_attn_kernel(
    const float* __restrict__ qkv, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
    int D, int pos, int text_len, float scale, uint16_t* __restrict__ out16) {
  extern __shared__ float psm[];
  float* rec = psm + kSlots * slot_floats<HD>();  // [nch][rec_floats]
  const int q = blockIdx.x, h = blockIdx.y;
  const int n = pos + max(text_len, q + 1);
  const int nch = (n + kChunk - 1) / kChunk;
  const float* qv = qkv + static_cast<size_t>(q) * 3 * D + h * HD;
  const int slot = threadIdx.x >> 6;
  for (int c = slot; c < nch; c += kSlots)
    attn_chunk_slot<HD>(qv, false, kc + h * HD, vc + h * HD, D, c * kChunk,
                        min(n, (c + 1) * kChunk), scale, psm + slot * slot_floats<HD>(), 1 + slot,
                        rec + c * rec_floats<HD>());
  __syncthreads();
  if (threadIdx.x < 32) {
    float o0, o1;
    attn_combine<HD>(rec, nch, false, &o0, &o1);
    out16[static_cast<size_t>(q) * D + h * HD + threadIdx.x] = f2h(o0);
    if (HD > 32) out16[static_cast<size_t>(q) * D + h * HD + 32 + threadIdx.x] = f2h(o1);
  }
}

// Standalone decode attention (gsvk_attention_decode): stage 1 computes one
// canonical 64-slot chunk record per (head, chunk) item, four items per CTA.
template <int HD>
__global__ void __launch_bounds__(kThreads) attn_chunks_kernel(
    const float* __restrict__ q, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
    int len, int H, int D, float scale, float* __restrict__ rec) {
  extern __shared__ float asm_[];
  const int nch = (len + kChunk - 1) / kChunk;
  const int slot = threadIdx.x >> 6;
  const int item = blockIdx.x * kSlots + slot;
  if (item >= H * nch) return;  // whole slot exits together (slot-local barriers only)
  const int h = item / nch, c = item - (item / nch) * nch;
  attn_chunk_slot<HD>(q + h * HD, true, kc + h * HD, vc + h * HD, D, c * kChunk,
                      min(len, (c + 1) * kChunk), scale, asm_ + slot * slot_floats<HD>(), 1 + slot,
                      rec + static_cast<size_t>(item) * rec_floats<HD>());
}

// Stage 2: one warp per head combines its chunk records in order.
template <int HD>
__global__ void attn_combine_kernel(const float* __restrict__ rec, int len, int H,
                                    float* __restrict__ out) {
  const int nch = (len + kChunk - 1) / kChunk;
  const int h = blockIdx.x;
  float o0, o1;
  attn_combine<HD>(rec + static_cast<size_t>(h) * nch * rec_floats<HD>(), nch, true, &o0, &o1);
  out[h * HD + threadIdx.x] = o0;
  if (HD > 32) out[h * HD + 32 + threadIdx.x] = o1;
}

// Row LayerNorm (kern.cpp:27-58, canonical order) writing fp32 and fp16.
__global__ void __launch_bounds__(256) ln_rows_canon_kernel(
    const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ b,
    float* __restrict__ y, uint16_t* __restrict__ y16, int n, double eps) {
  __shared__ float scratch[32];
  __shared__ float buf[4096];
  const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) buf[i] = xr[i];
  __syncthreads();
  ln_canon(buf, g, b, n, eps, scratch);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    y[static_cast<size_t>(blockIdx.x) * n + i] = buf[i];
    y16[static_cast<size_t>(blockIdx.x) * n + i] = f2h(buf[i]);
  }
}

int canon_gemm(const uint16_t* A, int lda, const uint16_t* B, int ldb, int M, int N, int K,
               const float* bias, int relu, const float* res, int ldr, float* c32, int ldc,
               uint16_t* c16, int ldc16, cudaStream_t st) {
  const long long warps = static_cast<long long>((M + 3) / 4) * ((N + 3) / 4);
  canon_gemm_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, st>>>(
      A, lda, B, ldb, M, N, K, bias, relu, res, ldr, c32, ldc, c16, ldc16);
  return check_launch("canon_gemm_kernel");
}
__global__ void rstd_check_kernel(const double* __restrict__ v, float* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = rstd_f32(v[i]);
}

}  // namespace

// --------------------------------------------------------------- host engine
struct T2SEngine {
  int L, D, H, F, V, cap;
  float eps, alpha;
  T2SDev dev{};
  int G = 0;                 // decode CTAs
  int HD = 0;
  DecodeArgs plan{};
  size_t decode_smem = 0;
  size_t attn_smem = 0;      // prefill attention dynamic shared memory
  const void* decode_fn = nullptr;
  const void* attn_fn = nullptr;
  // single-cluster decode (t2s_cluster_kernel): usable on this shape / GPU,
  // and which decode kernel gsvk_t2s_decode launches (1 grid, 2 cluster)
  bool cluster_ok = false;
  size_t cluster_smem = 0;
  int decode_kind = 1;
  // per-head cluster data-flow decode (t2s_flow_kernel): kind 3
  bool flow_ok = false;
  const void* flow_fn = nullptr;
  size_t flow_smem = 0;
  int flow_grid = 0;         // clusters x CTAs per cluster
  FlowArgs flow{};
  CUtensorMap flow_tk{}, flow_tv{};
  uint32_t flow_epoch = 1;   // exchange epochs used so far (never reused)
  gsvk_t2s_sampling sampling{};  // mode 0: greedy
  size_t flow_xbytes = 0;    // exchange words (zeroed at create)
  // device allocations
  void* weights = nullptr;   // one block: all fp16 weights + fp32 vectors + PE table
  void* w2_lanes = nullptr;  // W2 permuted for the single-cluster decode
  void* scratch = nullptr;
  int32_t* d_prompt = nullptr;
  int32_t* d_tokens = nullptr;
  int* d_nout = nullptr;
  float* d_margins = nullptr;
  unsigned long long* d_trace = nullptr;
  bool trace_on = false;
  // prefill buffers
  float *px = nullptr, *pqkv = nullptr, *phpre = nullptr;
  uint16_t *px16 = nullptr, *pattn16 = nullptr, *pff16 = nullptr;
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// PE row as the reference computes it (t2s_engine.cpp:711-720).
void pe_row_host(int D, size_t pos, float* pe) {
  const float log_inc = static_cast<float>(-std::log(10000.0) / static_cast<double>(D));
  const float p = static_cast<float>(pos);
  for (int d = 0; d < D; d += 2) {
    const float div = std::exp(static_cast<float>(d) * log_inc);
    pe[d] = std::sin(p * div);
    pe[d + 1] = std::cos(p * div);
  }
}

}  // namespace

}  // namespace gsvk

using namespace gsvk;

struct gsvk_t2s : gsvk::T2SEngine {};

namespace {
// gsvk_set_spin_limit_for_test: 0 = the kernels' own budgets.
uint32_t& test_spin_limit() {
  static uint32_t v = 0;
  return v;
}
}  // namespace

namespace {

// Decode launch plan for G persistent CTAs: weight slices sized for the
// largest CTA (rows / G rounded up), two layer buffers and the persistent
// logits slice in shared memory.  Sets e->G on success.
int decode_plan(gsvk_t2s* e, int G) {
  const int D = e->D, F = e->F, V = e->V, HD = e->HD;
  auto ceil_rows = [&](int rows) { return (rows + G - 1) / G; };
  DecodeArgs a = e->plan;
  a.mq = ceil_rows(3 * D);
  a.mo = ceil_rows(D);
  a.m1 = ceil_rows(F);
  a.m2 = ceil_rows(D);
  a.ml = ceil_rows(V);
  a.ln_off = static_cast<uint32_t>(align_up(
      ((size_t)a.mq * D + (size_t)a.mo * D + (size_t)a.m1 * D + (size_t)a.m2 * F) * 2, 16));
  a.layer_bytes = static_cast<uint32_t>(align_up((size_t)a.ln_off + (size_t)4 * D * 4, 128));
  const size_t slot_f = (size_t)kSlots * (HD == 32 ? slot_floats<32>() : slot_floats<64>());
  const size_t floats = slot_f + (size_t)D * 2 + std::max(D, F) + kChunk + 64;
  const size_t bias_f = align_up((size_t)a.mq + a.mo + a.m1 + a.m2, 4);
  const size_t smem = 128 + 2 * (size_t)a.layer_bytes + (size_t)a.ml * D * 2 + (size_t)2 * D * 4 +
                      floats * 4 + 8 * 4 + 4 * 8 + bias_f * 4 + align_up(V, 16) + 64;
  int dev = 0;
  cudaGetDevice(&dev);
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (smem > (size_t)max_optin)
    return fail(GSVK_ERR_UNSUPPORTED, "t2s decode on %d CTAs needs %zu B shared memory", G, smem);
  if (int rc = check_cuda(cudaFuncSetAttribute(e->decode_fn,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                          "cudaFuncSetAttribute(t2s_decode)"))
    return rc;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, e->decode_fn, kThreads, smem);
  if (per_sm < 1) return fail(GSVK_ERR_UNSUPPORTED, "t2s decode kernel does not fit an SM");
  e->plan = a;
  e->decode_smem = smem;
  e->G = G;
  return GSVK_OK;
}

// Per-head cluster decode (t2s_flow_kernel): one cluster of cs CTAs per head
// plus helper clusters of the same size for the grid-wide rows.  All clusters
// must be resident at once (the kernel's waits need co-resident CTAs), so for
// each cluster size the GPU's own count of simultaneously active clusters
// bounds the grid.  Among the sizes whose shared-memory plan fits, the one
// whose clusters cover a full cache's softmax chunks in the fewest rounds is
// taken, then the one with the most CTAs, then the largest (fewer q/k/v rows
// per CTA).  Leaves flow_ok false when none fits.
void flow_plan(gsvk_t2s* e, int max_optin) {
  const int D = e->D, F = e->F, V = e->V, H = e->H, HD = e->HD, sms = sm_count();
  const int vp = (V + 1) & ~1;
  if (D != kFlD || F % 2 || std::max(std::max(D, F), vp) > 2 * kThreads * kFlMaxPairs) return;
  const void* fn = HD == 32 ? (const void*)t2s_flow_kernel<32> : (const void*)t2s_flow_kernel<64>;
  int best_cs = 0, best_g = 0, best_rounds = 0;
  FlLayout best_y{};
  for (int cs = 8; cs >= 1; --cs) {
    if (cs * H > sms) continue;
    int nclust = std::min(sms / cs, D / cs);  // every CTA must own rows of every exchanged vector
    if (nclust < H) continue;
    FlLayout y = fl_layout(D, F, V, HD, cs, nclust * cs, e->cap);
    if (y.total > (uint32_t)max_optin || y.mq + y.mo + y.m1 + y.m2 > kThreads) continue;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)y.total) !=
        cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(nclust * cs);
    lc.blockDim = dim3(kThreads);
    lc.dynamicSmemBytes = y.total;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, fn, &lc) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    nclust = std::min(nclust, active);
    if (nclust < H) continue;
    // fewer clusters: the rows per CTA grow, so re-plan at the final grid
    y = fl_layout(D, F, V, HD, cs, nclust * cs, e->cap);
    if (y.total > (uint32_t)max_optin || y.mq + y.mo + y.m1 + y.m2 > kThreads) continue;
    // fewest attention rounds over a full cache first, then the most CTAs
    // (sizes are tried largest first, so ties keep the larger cluster)
    const int rounds = ((e->cap + kChunk - 1) / kChunk + cs * kSlots - 1) / (cs * kSlots);
    if (!best_cs || rounds < best_rounds || (rounds == best_rounds && nclust * cs > best_g)) {
      best_rounds = rounds;
      best_g = nclust * cs;
      best_cs = cs;
      best_y = y;
    }
  }
  if (!best_cs) return;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)best_y.total) !=
      cudaSuccess) {
    cudaGetLastError();
    return;
  }
  // K and V caches as 2-D tensors [L * cap rows][D] fp16; a box is one
  // head's HD columns of 64 consecutive slots (one softmax chunk)
  const uint64_t dims[2] = {(uint64_t)D, (uint64_t)e->L * e->cap};
  const uint64_t strides[1] = {(uint64_t)D * 2};
  const uint32_t box[2] = {(uint32_t)HD, (uint32_t)kChunk};
  if (encode_tiled(&e->flow_tk, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, e->dev.kc, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
      encode_tiled(&e->flow_tv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, e->dev.vc, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
    return;
  e->flow.cs = best_cs;
  e->flow.y = best_y;
  e->flow_grid = best_g;
  e->flow_fn = fn;
  e->flow_smem = best_y.total;
  e->flow_ok = true;
}

}  // namespace

extern "C" {

int gsvk_t2s_create(const gsvk_t2s_config* cfg, const gsvk_t2s_host_weights* w, gsvk_t2s_t* out) {
  if (!cfg || !w || !out) return fail(GSVK_ERR_INVALID, "t2s_create: null argument");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  const int L = cfg->n_layers, D = cfg->d_model, H = cfg->n_heads, F = cfg->ffn, V = cfg->vocab;
  const int cap = cfg->cap;
  if (L <= 0 || D <= 0 || H <= 0 || F <= 0 || V <= 1 || cap <= 0 || D % H != 0)
    return fail(GSVK_ERR_INVALID, "t2s_create: bad dimensions");
  const int HD = D / H;
  if ((HD != 32 && HD != 64) || D % 8 != 0 || F % 8 != 0 || D > 4096 || F > 16384)
    return fail(GSVK_ERR_UNSUPPORTED, "t2s_create: head_dim must be 32 or 64, D,F multiples of 8");
  if (cap > kMaxChunks * kChunk) return fail(GSVK_ERR_UNSUPPORTED, "t2s_create: cap too large");
  if (!w->wqkv || !w->bqkv || !w->wout || !w->bout || !w->w1 || !w->b1 || !w->w2 || !w->b2 ||
      !w->n1g || !w->n1b || !w->n2g || !w->n2b || !w->wpred || !w->audio_emb)
    return fail(GSVK_ERR_INVALID, "t2s_create: null weight");
  auto* e = new gsvk_t2s();
  e->L = L; e->D = D; e->H = H; e->F = F; e->V = V; e->cap = cap;
  e->eps = cfg->ln_eps; e->alpha = cfg->alpha_audio;

  // ---- weights: fp16 matrices, fp32 vectors, PE table (one allocation)
  const size_t nqkv = (size_t)L * 3 * D * D, nout = (size_t)L * D * D, n1 = (size_t)L * F * D,
               n2 = (size_t)L * D * F, npred = (size_t)V * D, nemb = (size_t)V * D;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
  const size_t o_wqkv = take(nqkv * 2), o_wout = take(nout * 2), o_w1 = take(n1 * 2),
               o_w2 = take(n2 * 2), o_pred = take(npred * 2), o_emb = take(nemb * 2);
  const size_t o_bqkv = take((size_t)L * 3 * D * 4), o_bout = take((size_t)L * D * 4),
               o_b1 = take((size_t)L * F * 4), o_b2 = take((size_t)L * D * 4),
               o_n1g = take((size_t)L * D * 4), o_n1b = take((size_t)L * D * 4),
               o_n2g = take((size_t)L * D * 4), o_n2b = take((size_t)L * D * 4),
               o_pe = take((size_t)cap * D * 4);
  if (cudaMalloc(&e->weights, off) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return fail(GSVK_ERR_NOMEM, "t2s_create: weights (%zu bytes)", off);
  }
  uint8_t* base = static_cast<uint8_t*>(e->weights);
  struct Up { size_t o; const void* src; size_t bytes; };
  std::vector<float> pe((size_t)cap * D);
  for (int p = 0; p < cap; ++p) pe_row_host(D, p, pe.data() + (size_t)p * D);
  const Up ups[] = {{o_wqkv, w->wqkv, nqkv * 2}, {o_wout, w->wout, nout * 2}, {o_w1, w->w1, n1 * 2},
                    {o_w2, w->w2, n2 * 2}, {o_pred, w->wpred, npred * 2}, {o_emb, w->audio_emb, nemb * 2},
                    {o_bqkv, w->bqkv, (size_t)L * 3 * D * 4}, {o_bout, w->bout, (size_t)L * D * 4},
                    {o_b1, w->b1, (size_t)L * F * 4}, {o_b2, w->b2, (size_t)L * D * 4},
                    {o_n1g, w->n1g, (size_t)L * D * 4}, {o_n1b, w->n1b, (size_t)L * D * 4},
                    {o_n2g, w->n2g, (size_t)L * D * 4}, {o_n2b, w->n2b, (size_t)L * D * 4},
                    {o_pe, pe.data(), (size_t)cap * D * 4}};
  for (const Up& u : ups) {
    int rc = check_cuda(cudaMemcpy(base + u.o, u.src, u.bytes, cudaMemcpyHostToDevice), "t2s upload");
    if (rc) { gsvk_t2s_destroy(e); return rc; }
  }
  T2SDev& d = e->dev;
  d.L = L; d.D = D; d.H = H; d.F = F; d.V = V; d.cap = cap; d.HD = HD;
  d.eps = cfg->ln_eps; d.alpha = cfg->alpha_audio;
  d.scale = 1.0f / std::sqrt(static_cast<float>(HD));
  d.wqkv = reinterpret_cast<const uint16_t*>(base + o_wqkv);
  d.wout = reinterpret_cast<const uint16_t*>(base + o_wout);
  d.w1 = reinterpret_cast<const uint16_t*>(base + o_w1);
  d.w2 = reinterpret_cast<const uint16_t*>(base + o_w2);
  d.wpred = reinterpret_cast<const uint16_t*>(base + o_pred);
  d.emb = reinterpret_cast<const uint16_t*>(base + o_emb);
  d.bqkv = reinterpret_cast<const float*>(base + o_bqkv);
  d.bout = reinterpret_cast<const float*>(base + o_bout);
  d.b1 = reinterpret_cast<const float*>(base + o_b1);
  d.b2 = reinterpret_cast<const float*>(base + o_b2);
  d.n1g = reinterpret_cast<const float*>(base + o_n1g);
  d.n1b = reinterpret_cast<const float*>(base + o_n1b);
  d.n2g = reinterpret_cast<const float*>(base + o_n2g);
  d.n2b = reinterpret_cast<const float*>(base + o_n2b);
  d.pe = reinterpret_cast<const float*>(base + o_pe);

  // ---- KV cache + decode scratch + prefill buffers (one allocation)
  off = 0;
  const size_t o_kc = take((size_t)L * cap * D * 2), o_vc = take((size_t)L * cap * D * 2),
               o_q = take((size_t)D * 4), o_part = take((size_t)H * kMaxChunks * (HD + 4) * 4),
               o_hpre = take((size_t)D * 4), o_ff = take((size_t)F * 4), o_xpre = take((size_t)D * 4),
               o_logits = take((size_t)V * 4), o_bar = take(256), o_prompt = take((size_t)cap * 4),
               o_tok = take((size_t)cap * 4), o_nout = take(256), o_marg = take((size_t)cap * 4),
               o_px = take((size_t)cap * D * 4), o_pqkv = take((size_t)cap * 3 * D * 4),
               o_phpre = take((size_t)cap * D * 4), o_px16 = take((size_t)cap * D * 2),
               o_pattn = take((size_t)cap * D * 2), o_pff = take((size_t)cap * F * 2),
               o_trace = take((size_t)kTraceSteps * kTraceStride * 8),
               o_attn = take((size_t)D * 4), o_ticket = take((size_t)H * 4);
  const int vp = (V + 1) & ~1;
  const size_t o_xattn = take((size_t)2 * D * 8), o_xhpre = take((size_t)2 * D * 8),
               o_xff = take((size_t)2 * F * 8), o_xxpre = take((size_t)2 * D * 8),
               o_xlog = take((size_t)2 * vp * 8);
  if (cudaMalloc(&e->scratch, off) != cudaSuccess) {
    cudaGetLastError();
    gsvk_t2s_destroy(e);
    return fail(GSVK_ERR_NOMEM, "t2s_create: scratch (%zu bytes)", off);
  }
  uint8_t* sb = static_cast<uint8_t*>(e->scratch);
  if (int rc = check_cuda(cudaMemset(sb, 0, off), "t2s scratch memset")) {
    gsvk_t2s_destroy(e);
    return rc;
  }
  d.kc = reinterpret_cast<uint16_t*>(sb + o_kc);
  d.vc = reinterpret_cast<uint16_t*>(sb + o_vc);
  d.q = reinterpret_cast<float*>(sb + o_q);
  d.part = reinterpret_cast<float*>(sb + o_part);
  d.hpre = reinterpret_cast<float*>(sb + o_hpre);
  d.ff = reinterpret_cast<float*>(sb + o_ff);
  d.xpre = reinterpret_cast<float*>(sb + o_xpre);
  d.logits = reinterpret_cast<float*>(sb + o_logits);
  d.bar = reinterpret_cast<unsigned*>(sb + o_bar);
  d.attn = reinterpret_cast<float*>(sb + o_attn);
  d.ticket = reinterpret_cast<unsigned*>(sb + o_ticket);
  d.status = device_status();
  e->d_prompt = reinterpret_cast<int32_t*>(sb + o_prompt);
  e->d_tokens = reinterpret_cast<int32_t*>(sb + o_tok);
  e->d_nout = reinterpret_cast<int*>(sb + o_nout);
  e->d_margins = reinterpret_cast<float*>(sb + o_marg);
  e->px = reinterpret_cast<float*>(sb + o_px);
  e->pqkv = reinterpret_cast<float*>(sb + o_pqkv);
  e->phpre = reinterpret_cast<float*>(sb + o_phpre);
  e->px16 = reinterpret_cast<uint16_t*>(sb + o_px16);
  e->pattn16 = reinterpret_cast<uint16_t*>(sb + o_pattn);
  e->pff16 = reinterpret_cast<uint16_t*>(sb + o_pff);
  e->d_trace = reinterpret_cast<unsigned long long*>(sb + o_trace);
  e->flow.xattn = reinterpret_cast<uint64_t*>(sb + o_xattn);
  e->flow.xhpre = reinterpret_cast<uint64_t*>(sb + o_xhpre);
  e->flow.xff = reinterpret_cast<uint64_t*>(sb + o_xff);
  e->flow.xxpre = reinterpret_cast<uint64_t*>(sb + o_xxpre);
  e->flow.xlog = reinterpret_cast<uint64_t*>(sb + o_xlog);
  e->flow.vp = vp;
  e->flow_xbytes = o_xlog + (size_t)2 * vp * 8 - o_xattn;

  // ---- decode launch plan (one CTA per SM by default) and prefill attention
  const size_t slot_f = (size_t)kSlots * (HD == 32 ? slot_floats<32>() : slot_floats<64>());
  const size_t max_nch = ((size_t)cap + kChunk - 1) / kChunk;
  e->attn_smem = (slot_f + max_nch * (HD + 4)) * 4;
  e->HD = HD;
  e->decode_fn = HD == 32 ? (const void*)t2s_decode_kernel<32> : (const void*)t2s_decode_kernel<64>;
  e->attn_fn = HD == 32 ? (const void*)prefill_attn_kernel<32> : (const void*)prefill_attn_kernel<64>;
  int dev = 0;
  cudaGetDevice(&dev);
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e->attn_smem > (size_t)max_optin) {
    gsvk_t2s_destroy(e);
    return fail(GSVK_ERR_UNSUPPORTED, "t2s prefill attention needs %zu B shared memory", e->attn_smem);
  }
  if (int rc = check_cuda(cudaFuncSetAttribute(e->attn_fn,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)e->attn_smem),
                          "cudaFuncSetAttribute(prefill_attn)")) {
    gsvk_t2s_destroy(e);
    return rc;
  }
  if (int rc = decode_plan(e, sm_count())) {
    gsvk_t2s_destroy(e);
    return rc;
  }
  // W2 in lane order (both decode kernels read it when F = kClF)
  if (F == kClF) {
    const size_t w2_bytes = (size_t)L * D * F * 2;
    if (cudaMalloc(&e->w2_lanes, w2_bytes) != cudaSuccess) {
      cudaGetLastError();
      gsvk_t2s_destroy(e);
      return fail(GSVK_ERR_NOMEM, "t2s_create: lane-ordered W2 (%zu bytes)", w2_bytes);
    }
    uint16_t* dst = static_cast<uint16_t*>(e->w2_lanes);
    w2_lane_order_kernel<<<(unsigned)((size_t)L * D), 256>>>(d.w2, dst);
    if (int rc = check_cuda(cudaDeviceSynchronize(), "t2s_create: W2 lane order")) {
      gsvk_t2s_destroy(e);
      return rc;
    }
    d.w2p = dst;
  }
  // single-cluster decode: the configuration's shape (d 512, head 32, ffn
  // 2048), at most one head per CTA, chunk records for the whole cache in
  // shared memory, and a GPU that can place a 16-CTA cluster of this size
  if (HD == kClHD && D == kClD && F == kClF && H <= kClCS && cap <= kClMaxChunks * kChunk) {
    const size_t smem = cl_layout(V).total;
    const void* fn = (const void*)t2s_cluster_kernel;
    if (smem <= (size_t)max_optin &&
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
            cudaSuccess &&
        cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t lc{};
      lc.gridDim = dim3(kClCS);
      lc.blockDim = dim3(kClThreads);
      lc.dynamicSmemBytes = smem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = kClCS;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      lc.attrs = at;
      lc.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, fn, &lc) == cudaSuccess && clusters >= 1 &&
          d.w2p) {
        e->cluster_ok = true;
        e->cluster_smem = smem;
      }
    }
    cudaGetLastError();  // a refused attribute or query only disables the variant
  }
  flow_plan(e, max_optin);
  // the per-head cluster decode when this shape and GPU can run it
  e->decode_kind = e->flow_ok ? 3 : 1;
  *out = e;
  return GSVK_OK;
}

int gsvk_t2s_destroy(gsvk_t2s_t h) {
  if (!h) return GSVK_OK;
  if (h->weights) cudaFree(h->weights);
  if (h->w2_lanes) cudaFree(h->w2_lanes);
  if (h->scratch) cudaFree(h->scratch);
  delete h;
  return GSVK_OK;
}

int gsvk_t2s_load_kv(gsvk_t2s_t h, const uint16_t* k_host, const uint16_t* v_host, size_t prefix,
                     size_t src_rows, gsvk_stream_t stream) {
  if (!h || (prefix && (!k_host || !v_host))) return fail(GSVK_ERR_INVALID, "t2s_load_kv: null");
  if (prefix > (size_t)h->cap || src_rows < prefix)
    return fail(GSVK_ERR_INVALID, "t2s_load_kv: prefix %zu exceeds cache", prefix);
  const size_t row = (size_t)h->D * 2;
  for (int l = 0; l < h->L && prefix; ++l) {
    int rc = check_cuda(cudaMemcpyAsync(h->dev.kc + (size_t)l * h->cap * h->D,
                                        k_host + (size_t)l * src_rows * h->D, prefix * row,
                                        cudaMemcpyDefault, as_cuda(stream)),
                        "t2s_load_kv k");
    if (rc) return rc;
    rc = check_cuda(cudaMemcpyAsync(h->dev.vc + (size_t)l * h->cap * h->D,
                                    v_host + (size_t)l * src_rows * h->D, prefix * row,
                                    cudaMemcpyDefault, as_cuda(stream)),
                    "t2s_load_kv v");
    if (rc) return rc;
  }
  return GSVK_OK;
}

int gsvk_t2s_prefill(gsvk_t2s_t h, float* x, size_t S, size_t pos, size_t text_len,
                     gsvk_stream_t stream) {
  if (!h || !x || S == 0) return fail(GSVK_ERR_INVALID, "t2s_prefill: null or empty");
  if (pos + S > (size_t)h->cap) return fail(GSVK_ERR_INVALID, "t2s_prefill: exceeds cache");
  const T2SDev& d = h->dev;
  const int D = h->D, F = h->F;
  cudaStream_t st = as_cuda(stream);
  int rc = gsvk_f32_to_f16(x, h->px16, S * D, stream);
  if (rc) return rc;
  for (int l = 0; l < h->L; ++l) {
    // QKV: qkv = f16(x) . Wqkv^T + b
    if ((rc = canon_gemm(h->px16, D, d.wqkv + (size_t)l * 3 * D * D, D, (int)S, 3 * D, D,
                         d.bqkv + (size_t)l * 3 * D, 0, nullptr, 0, h->pqkv, 3 * D, nullptr, 0, st)))
      return rc;
    uint16_t* kl = d.kc + (size_t)l * h->cap * D;
    uint16_t* vl = d.vc + (size_t)l * h->cap * D;
    kv_append_kernel<<<(unsigned)S, 256, 0, st>>>(h->pqkv, (int)S, D, kl, vl, (int)pos);
    if ((rc = check_launch("kv_append_kernel"))) return rc;
    {
      dim3 grid((unsigned)S, (unsigned)h->H);
      int Di = D, posi = (int)pos, tl = (int)text_len;
      float sc = d.scale;
      const float* qkv = h->pqkv;
      uint16_t* o16 = h->pattn16;
      void* args[] = {&qkv, &kl, &vl, &Di, &posi, &tl, &sc, &o16};
      if ((rc = check_cuda(cudaLaunchKernel(h->attn_fn, grid, dim3(kThreads), args, h->attn_smem, st),
                           "prefill_attn_kernel")))
        return rc;
    }
    // out-proj + bias + residual(x) -> hpre ; x = LN1(hpre)
    if ((rc = canon_gemm(h->pattn16, D, d.wout + (size_t)l * D * D, D, (int)S, D, D,
                         d.bout + (size_t)l * D, 0, x, D, h->phpre, D, nullptr, 0, st)))
      return rc;
    ln_rows_canon_kernel<<<(unsigned)S, kThreads, 0, st>>>(h->phpre, d.n1g + (size_t)l * D,
                                                         d.n1b + (size_t)l * D, x, h->px16, D, h->eps);
    if ((rc = check_launch("ln_rows_canon_kernel"))) return rc;
    // FFN: ff16 = relu(f16(x) . W1^T + b1) ; hpre = f16(ff) . W2^T + b2 + x ; x = LN2(hpre)
    if ((rc = canon_gemm(h->px16, D, d.w1 + (size_t)l * F * D, D, (int)S, F, D,
                         d.b1 + (size_t)l * F, 1, nullptr, 0, nullptr, 0, h->pff16, F, st)))
      return rc;
    if ((rc = canon_gemm(h->pff16, F, d.w2 + (size_t)l * D * F, F, (int)S, D, F,
                         d.b2 + (size_t)l * D, 0, x, D, h->phpre, D, nullptr, 0, st)))
      return rc;
    ln_rows_canon_kernel<<<(unsigned)S, kThreads, 0, st>>>(h->phpre, d.n2g + (size_t)l * D,
                                                         d.n2b + (size_t)l * D, x, h->px16, D, h->eps);
    if ((rc = check_launch("ln_rows_canon_kernel"))) return rc;
  }
  return GSVK_OK;
}

int gsvk_t2s_prompt(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_dev, size_t P,
                    gsvk_stream_t stream) {
  if (!h || !prompt_dev || P == 0) return fail(GSVK_ERR_INVALID, "t2s_prompt: null or empty");
  if (prefix + P > (size_t)h->cap)
    return fail(GSVK_ERR_INVALID, "t2s_prompt: prefix+P=%zu exceeds cap %d", prefix + P, h->cap);
  const T2SDev& d = h->dev;
  cudaStream_t st = as_cuda(stream);
  const int D = h->D;
  embed_kernel<<<(unsigned)P, 256, 0, st>>>(prompt_dev, (int)P, d.emb, d.pe, 0, h->alpha, D, h->px,
                                           h->px16);
  int rc = check_launch("embed_kernel");
  if (rc) return rc;
  if ((rc = gsvk_t2s_prefill(h, h->px, P, prefix, 0, stream))) return rc;
  // first logits from the last prompt row, fp32 activations (t2s_engine.cpp:703-707, 1806)
  canon_gemv_kernel<<<(unsigned)((h->V * 32 + 255) / 256), 256, 0, st>>>(
      d.wpred, h->px + (P - 1) * D, d.logits, h->V, D);
  return check_launch("canon_gemv_kernel");
}

int gsvk_t2s_decode(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_dev, size_t P,
                    size_t max_steps, int stop_on_eos, int32_t* tokens_dev, int* n_out_dev,
                    float* margins_dev, gsvk_stream_t stream) {
  if (!h || !prompt_dev || P == 0 || !tokens_dev || !n_out_dev)
    return fail(GSVK_ERR_INVALID, "t2s_decode: null argument or empty prompt");
  if (prefix + P + max_steps > (size_t)h->cap)
    return fail(GSVK_ERR_INVALID, "t2s_decode: prefix+P+steps=%zu exceeds cap %d",
                prefix + P + max_steps, h->cap);
  const T2SDev& d = h->dev;
  cudaStream_t st = as_cuda(stream);
  int rc;
  if ((rc = check_cuda(cudaMemsetAsync(d.bar, 0, 4, st), "reset grid barrier"))) return rc;
  if ((rc = check_cuda(cudaMemsetAsync(d.ticket, 0, (size_t)d.H * 4, st), "reset head tickets")))
    return rc;
  if ((rc = check_cuda(cudaMemsetAsync(n_out_dev, 0, 4, st), "reset n_out"))) return rc;
  if (max_steps == 0) return GSVK_OK;
  DecodeArgs a = h->plan;
  a.pos0 = (int)(prefix + P);
  a.pe0 = (int)P;
  a.max_steps = (int)max_steps;
  a.stop_on_eos = stop_on_eos;
  a.hist = prompt_dev;
  a.n_hist = (int)P;
  a.tokens = tokens_dev;
  a.n_out = n_out_dev;
  a.margins = margins_dev;
  a.trace = h->trace_on ? h->d_trace : nullptr;
  a.samp_mode = h->sampling.mode;
  a.samp_top_k = h->sampling.top_k;
  a.samp_top_p = h->sampling.top_p;
  a.samp_temp = h->sampling.temperature;
  a.samp_pen = h->sampling.rep_penalty;
  a.samp_seed = h->sampling.seed;
  if (a.samp_mode == 1) {
    if (h->decode_kind != 3)
      return fail(GSVK_ERR_UNSUPPORTED, "t2s_decode: top-k sampling runs on decode kernel 3 only");
    if (a.samp_seed == 0)  // the reference draws a fresh seed (std::random_device)
      a.samp_seed = static_cast<unsigned long long>(
          std::chrono::high_resolution_clock::now().time_since_epoch().count()) | 1ull;
  }
  T2SDev dv = d;
  if (h->decode_kind == 3) {
    // this launch's exchange epochs: epoch0 + 1 .. epoch0 + steps * (L + 1);
    // near the end of the 32-bit range the words are cleared and epochs restart
    const uint64_t need = (uint64_t)max_steps * (h->L + 1) + 2;
    if ((uint64_t)h->flow_epoch + need >= 0xFFFFFFF0ull) {
      if ((rc = check_cuda(cudaMemsetAsync(h->flow.xattn, 0, h->flow_xbytes, st),
                           "reset exchange words")))
        return rc;
      h->flow_epoch = 1;
    }
    FlowArgs fa = h->flow;
    fa.epoch0 = h->flow_epoch;
    fa.spin = test_spin_limit() ? test_spin_limit() : kFlSpin;
    h->flow_epoch += (uint32_t)need;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(h->flow_grid);
    lc.blockDim = dim3(kThreads);
    lc.dynamicSmemBytes = h->flow_smem;
    lc.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = fa.cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    if (h->HD == 32)
      return check_cuda(cudaLaunchKernelEx(&lc, t2s_flow_kernel<32>, dv, a, fa, h->flow_tk, h->flow_tv),
                        "t2s_flow_kernel (cluster launch)");
    return check_cuda(cudaLaunchKernelEx(&lc, t2s_flow_kernel<64>, dv, a, fa, h->flow_tk, h->flow_tv),
                      "t2s_flow_kernel (cluster launch)");
  }
  if (h->decode_kind == 2) {
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(kClCS);
    lc.blockDim = dim3(kClThreads);
    lc.dynamicSmemBytes = h->cluster_smem;
    lc.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kClCS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&lc, t2s_cluster_kernel, dv, a),
                      "t2s_cluster_kernel (cluster launch)");
  }
  void* args[] = {&dv, &a};
  return check_cuda(cudaLaunchCooperativeKernel(h->decode_fn, dim3(h->G), dim3(kThreads),
                                                args, h->decode_smem, st),
                    "t2s_decode_kernel (cooperative launch)");
}

int gsvk_t2s_set_decode_kernel(gsvk_t2s_t h, int kind) {
  if (!h) return fail(GSVK_ERR_INVALID, "t2s_set_decode_kernel: null handle");
  if (kind < 0 || kind > 3) return fail(GSVK_ERR_INVALID, "t2s_set_decode_kernel: kind %d", kind);
  if (kind == 2 && !h->cluster_ok)
    return fail(GSVK_ERR_UNSUPPORTED, "t2s_set_decode_kernel: the single-cluster decode does not "
                                      "fit this model shape or GPU");
  if (kind == 3 && !h->flow_ok)
    return fail(GSVK_ERR_UNSUPPORTED, "t2s_set_decode_kernel: the per-head cluster decode does not "
                                      "fit this model shape or GPU");
  h->decode_kind = kind == 0 ? (h->flow_ok ? 3 : 1) : kind;
  return GSVK_OK;
}

int gsvk_t2s_decode_kernel(gsvk_t2s_t h) { return h ? h->decode_kind : 0; }

int gsvk_set_spin_limit_for_test(uint32_t polls) {
  test_spin_limit() = polls;
  return GSVK_OK;
}

int gsvk_test_rstd(const double* v, float* out, size_t n, gsvk_stream_t stream) {
  if (!v || !out || !n) return fail(GSVK_ERR_INVALID, "test_rstd: null pointer or zero size");
  if (n > 0x7fffffffu) return fail(GSVK_ERR_UNSUPPORTED, "test_rstd: n too large");
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  rstd_check_kernel<<<blocks, 256, 0, as_cuda(stream)>>>(v, out, static_cast<int>(n));
  if (int rc = check_launch("rstd_check_kernel")) return rc;
  return check_cuda(cudaStreamSynchronize(as_cuda(stream)), "test_rstd");
}

int gsvk_t2s_set_sampling(gsvk_t2s_t h, const gsvk_t2s_sampling* sp) {
  if (!h) return fail(GSVK_ERR_INVALID, "t2s_set_sampling: null handle");
  if (!sp) {
    h->sampling = gsvk_t2s_sampling{};
    return GSVK_OK;
  }
  if (sp->mode != 0 && sp->mode != 1)
    return fail(GSVK_ERR_INVALID, "t2s_set_sampling: mode %d (0 greedy, 1 top-k)", sp->mode);
  if (sp->mode == 1) {
    if (sp->top_k < 1 || !(sp->top_p > 0.f && sp->top_p <= 1.f) || !(sp->rep_penalty > 0.f) ||
        sp->temperature != sp->temperature)
      return fail(GSVK_ERR_INVALID, "t2s_set_sampling: top_k >= 1, 0 < top_p <= 1, "
                                    "rep_penalty > 0 and a temperature are required");
    if (!h->flow_ok)
      return fail(GSVK_ERR_UNSUPPORTED, "t2s_set_sampling: top-k sampling runs on decode kernel "
                                        "3, which this shape or GPU cannot run");
  }
  h->sampling = *sp;
  return GSVK_OK;
}

int gsvk_t2s_set_decode_ctas(gsvk_t2s_t h, int ctas) {
  if (!h) return fail(GSVK_ERR_INVALID, "t2s_set_decode_ctas: null handle");
  const int sms = sm_count();
  if (ctas < 0 || ctas > sms)
    return fail(GSVK_ERR_INVALID, "t2s_set_decode_ctas: %d CTAs (0 or 1..%d)", ctas, sms);
  return decode_plan(h, ctas == 0 ? sms : ctas);
}

int gsvk_t2s_generate_device(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_dev, size_t P,
                             size_t max_steps, int stop_on_eos, int32_t* tokens_dev,
                             int* n_out_dev, float* margins_dev, gsvk_stream_t stream) {
  if (!h || !prompt_dev || P == 0 || !tokens_dev || !n_out_dev)
    return fail(GSVK_ERR_INVALID, "t2s_generate: null argument or empty prompt");
  if (prefix + P + max_steps > (size_t)h->cap)
    return fail(GSVK_ERR_INVALID, "t2s_generate: prefix+P+steps=%zu exceeds cap %d",
                prefix + P + max_steps, h->cap);
  int rc = gsvk_t2s_prompt(h, prefix, prompt_dev, P, stream);
  if (rc) return rc;
  return gsvk_t2s_decode(h, prefix, prompt_dev, P, max_steps, stop_on_eos, tokens_dev, n_out_dev,
                         margins_dev, stream);
}

int gsvk_t2s_launches_per_generate(gsvk_t2s_t h) {
  // embed + per layer (4 GEMMs, KV append, attention, 2 LayerNorms) + logits
  // GEMV + the decode kernel
  return h ? 1 + 8 * h->L + 1 + 1 : 0;
}

int gsvk_t2s_generate(gsvk_t2s_t h, size_t prefix, const int32_t* prompt_host, size_t P,
                      size_t max_steps, int stop_on_eos, int32_t* tokens_host, float* margins_host,
                      int* n_out, gsvk_stream_t stream) {
  if (!h || !prompt_host || !tokens_host || !n_out) return fail(GSVK_ERR_INVALID, "t2s_generate: null");
  if (P > (size_t)h->cap) return fail(GSVK_ERR_INVALID, "t2s_generate: prompt longer than cache");
  cudaStream_t st = as_cuda(stream);
  int rc = check_cuda(cudaMemcpyAsync(h->d_prompt, prompt_host, P * 4, cudaMemcpyHostToDevice, st),
                      "prompt upload");
  if (rc) return rc;
  rc = gsvk_t2s_generate_device(h, prefix, h->d_prompt, P, max_steps, stop_on_eos, h->d_tokens,
                                h->d_nout, margins_host ? h->d_margins : nullptr, stream);
  if (rc) return rc;
  int n = 0;
  if ((rc = check_cuda(cudaMemcpyAsync(&n, h->d_nout, 4, cudaMemcpyDeviceToHost, st), "n_out")))
    return rc;
  if ((rc = check_cuda(cudaStreamSynchronize(st), "t2s_generate sync"))) return rc;
  if (n < 0 || (size_t)n > max_steps) return fail(GSVK_ERR_CUDA, "t2s_generate: bad count %d", n);
  *n_out = n;
  if (n && (rc = check_cuda(cudaMemcpy(tokens_host, h->d_tokens, (size_t)n * 4,
                                       cudaMemcpyDeviceToHost), "tokens download")))
    return rc;
  if (margins_host && max_steps &&
      (rc = check_cuda(cudaMemcpy(margins_host, h->d_margins, max_steps * 4, cudaMemcpyDeviceToHost),
                       "margins download")))
    return rc;
  return gsvk_device_status(1);
}

int gsvk_t2s_set_trace(gsvk_t2s_t h, int enable) {
  if (!h) return fail(GSVK_ERR_INVALID, "t2s_set_trace: null handle");
  h->trace_on = enable != 0;
  if (h->trace_on)
    return check_cuda(cudaMemset(h->d_trace, 0, (size_t)kTraceSteps * kTraceStride * 8),
                      "trace reset");
  return GSVK_OK;
}

int gsvk_t2s_read_trace(gsvk_t2s_t h, unsigned long long* host_out, size_t n) {
  if (!h || !host_out) return fail(GSVK_ERR_INVALID, "t2s_read_trace: null");
  const size_t total = (size_t)kTraceSteps * kTraceStride;
  return check_cuda(cudaMemcpy(host_out, h->d_trace, (n < total ? n : total) * 8,
                               cudaMemcpyDeviceToHost),
                    "trace download");
}

int gsvk_t2s_read_kv(gsvk_t2s_t h, uint16_t* k_host, uint16_t* v_host) {
  if (!h || !k_host || !v_host) return fail(GSVK_ERR_INVALID, "t2s_read_kv: null");
  const size_t bytes = (size_t)h->L * h->cap * h->D * 2;
  int rc = check_cuda(cudaMemcpy(k_host, h->dev.kc, bytes, cudaMemcpyDeviceToHost), "kv download");
  if (rc) return rc;
  return check_cuda(cudaMemcpy(v_host, h->dev.vc, bytes, cudaMemcpyDeviceToHost), "kv download");
}

int gsvk_t2s_read_logits(gsvk_t2s_t h, float* host_out) {
  if (!h || !host_out) return fail(GSVK_ERR_INVALID, "t2s_read_logits: null");
  return check_cuda(cudaMemcpy(host_out, h->dev.logits, (size_t)h->V * 4, cudaMemcpyDeviceToHost),
                    "logits download");
}

size_t gsvk_attention_workspace_floats(size_t len, size_t n_heads, size_t head_dim) {
  return n_heads * ((len + kChunk - 1) / kChunk) * (head_dim + 4);
}

int gsvk_attention_decode(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                          size_t len, size_t n_heads, size_t head_dim, size_t row_stride,
                          float scale, float* out, float* workspace, gsvk_stream_t stream) {
  if (!q || !kcache || !vcache || !out || !workspace || len == 0 || n_heads == 0)
    return fail(GSVK_ERR_INVALID, "attention_decode: null pointer or zero size");
  if (head_dim != 32 && head_dim != 64)
    return fail(GSVK_ERR_UNSUPPORTED, "attention_decode: head_dim must be 32 or 64");
  // n_heads and row_stride are narrowed to int below: reject anything that
  // would not survive the cast (and keep n_heads * head_dim from wrapping).
  if (n_heads > (1u << 20) || row_stride > static_cast<size_t>(INT32_MAX))
    return fail(GSVK_ERR_INVALID, "attention_decode: n_heads or row stride out of range");
  if (row_stride < n_heads * head_dim || row_stride % 8 != 0 || len > (1u << 24))
    return fail(GSVK_ERR_INVALID, "attention_decode: bad row stride or length");
  if (!aligned16(q) || !aligned16(kcache) || !aligned16(vcache))
    return fail(GSVK_ERR_ALIGN, "attention_decode: q, K and V need 16-byte alignment");
  cudaStream_t st = as_cuda(stream);
  const int L = (int)len, H = (int)n_heads, D = (int)row_stride;
  const int items = H * ((L + kChunk - 1) / kChunk);
  const unsigned grid = (unsigned)((items + kSlots - 1) / kSlots);
  if (head_dim == 32) {
    const size_t sm = (size_t)kSlots * slot_floats<32>() * 4;
    attn_chunks_kernel<32><<<grid, kThreads, sm, st>>>(q, kcache, vcache, L, H, D, scale, workspace);
    int rc = check_launch("attn_chunks_kernel");
    if (rc) return rc;
    attn_combine_kernel<32><<<(unsigned)H, 32, 0, st>>>(workspace, L, H, out);
  } else {
    const size_t sm = (size_t)kSlots * slot_floats<64>() * 4;
    attn_chunks_kernel<64><<<grid, kThreads, sm, st>>>(q, kcache, vcache, L, H, D, scale, workspace);
    int rc = check_launch("attn_chunks_kernel");
    if (rc) return rc;
    attn_combine_kernel<64><<<(unsigned)H, 32, 0, st>>>(workspace, L, H, out);
  }
  return check_launch("attn_combine_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode attention.
//
// For callers that must not allocate device memory at all: code running
// under an external allocator that owns every byte of device memory (a host
// framework's memory pool, a fixed-budget embedded deployment), or code that
// may not touch the CUDA allocator on its call path.  The chunk records that
// gsvk_attention_decode keeps in a caller-provided workspace live here in a
// fixed file-scope device array instead.  Every GPU that loads this library
// holds this array (1 MiB) until the process exits.
namespace {

constexpr size_t kNoAllocAttnFloats = 262144;  // 1 MiB of fp32 chunk records
static __device__ __align__(256) float g_noalloc_attn_scratch[kNoAllocAttnFloats];

std::mutex g_noalloc_mu;
// Device address of the array, per device, and the driver context it was
// resolved in: an address is only valid in its own context, so a caller that
// switches to another context (or resets the device, which makes a new
// primary context) gets the address resolved again.
struct NoAllocSlot {
  void* ctx = nullptr;
  float* ptr = nullptr;
};
NoAllocSlot g_noalloc_slot[64];
using CtxGetCurrentFn = int (*)(void**);
CtxGetCurrentFn g_ctx_get_current = nullptr;

}  // namespace

extern "C" {

size_t gsvk_attention_decode_noalloc_max_floats(void) { return kNoAllocAttnFloats; }

int gsvk_attention_decode_noalloc(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                  size_t len, size_t n_heads, size_t head_dim, size_t row_stride,
                                  float scale, float* out, gsvk_stream_t stream) {
  if ((head_dim == 32 || head_dim == 64) && n_heads > 0) {
    // Compared by division so that no product can wrap past the limit.
    const size_t per_head = (len / kChunk + (len % kChunk != 0)) * (head_dim + 4);
    if (per_head > kNoAllocAttnFloats || n_heads > kNoAllocAttnFloats / per_head)
      return fail(GSVK_ERR_UNSUPPORTED,
                  "attention_decode_noalloc: needs more scratch than the static array holds "
                  "(%zu floats; n_heads * ceil(len/64) * (head_dim+4) must not exceed it)",
                  kNoAllocAttnFloats);
  }
  int dev = -1;
  int rc = check_cuda(cudaGetDevice(&dev), "attention_decode_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(GSVK_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  float* scratch = nullptr;
  {
    // One-time set-up per device, with that device current: host code cannot
    // use the array's name as a device address, so resolve it here.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_ctx_get_current) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult qr;
      rc = check_cuda(cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &qr),
                      "attention_decode_noalloc: cudaGetDriverEntryPoint");
      if (rc) return rc;
      if (qr != cudaDriverEntryPointSuccess || !fn)
        return fail(GSVK_ERR_NODEV, "attention_decode_noalloc: driver lacks cuCtxGetCurrent");
      g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    }
    void* ctx = nullptr;
    if (g_ctx_get_current(&ctx) != 0 || !ctx)
      return fail(GSVK_ERR_NODEV, "attention_decode_noalloc: no current CUDA context");
    NoAllocSlot& slot = g_noalloc_slot[dev];
    if (!slot.ptr || slot.ctx != ctx) {
      void* p = nullptr;
      rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_attn_scratch),
                      "attention_decode_noalloc: cudaGetSymbolAddress");
      if (rc) return rc;
      slot.ptr = static_cast<float*>(p);
      slot.ctx = ctx;
    }
    scratch = slot.ptr;
  }
  // Same kernels as gsvk_attention_decode; the records it reads are all
  // written earlier in the same call, so nothing needs clearing between calls.
  return gsvk_attention_decode(q, kcache, vcache, len, n_heads, head_dim, row_stride, scale, out,
                               scratch, stream);
}

}  // extern "C"
