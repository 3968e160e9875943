// t2s_flow.cuh — batch-1 T2S decode as a data-flow kernel over per-head
// thread-block clusters.  Included by t2s.cu inside its anonymous namespace
// (it shares T2SDev, DecodeArgs, the slot helpers and the canonical
// arithmetic of canon.cuh).
//
// t2s_decode_kernel separates the five phases of a layer by grid barriers
// and re-reads each phase's vector after the barrier: two L2 round trips
// plus the barrier's contention per phase.  Here:
//   * the grid is one cluster of `cs` CTAs per attention head.  A cluster
//     computes its head's q, k and v rows, pushes them into every member's
//     shared memory (distributed shared memory) and passes a hardware
//     cluster barrier; its members then run the head's 64-slot softmax
//     chunks from K/V tiles that TMA loaded into shared memory a layer
//     earlier, push the chunk records to the cluster's first CTA, pass a
//     second cluster barrier, and that CTA merges the records;
//   * vectors that every CTA needs (attention output, pre-LayerNorm rows,
//     FFN activations, layer output, logits) travel through global
//     "exchange words": one 64-bit store of {value, epoch} per element.  A
//     consumer polls the words themselves until each carries the exchange's
//     epoch, so the data and its readiness arrive in the same load (no
//     barrier, no second read).  Epochs never repeat within or across
//     launches, and every vector is double-buffered by epoch parity; every
//     CTA produces rows of every exchanged vector, so no producer can
//     overwrite a buffer before every consumer has read it;
//   * sampling is redundant in every CTA (identical logits, identical
//     decision); the first CTA of each cluster broadcasts its decision to
//     its members so that a cluster always takes the same number of
//     cluster barriers, even after a failed wait.
// Arithmetic is exactly t2s_decode_kernel's (same canonical dot products,
// chunked softmax, LayerNorm, rounding points): tokens, margins, logits and
// the KV cache are bit-identical to it and to the oracle.
//
// Every wait is bounded.  A poll that gives up (spin budget, or another CTA
// recorded a failure in the status word) marks this CTA failed; a failed
// CTA stops waiting but keeps the cluster's barrier sequence, and its
// cluster stops at the next step boundary.

constexpr uint32_t kFlSpin = 1u << 22;  // polls of one exchange word pair (seconds)
constexpr int kFlMaxPairs = 8;          // exchange vectors up to 8 x 2 x 256 = 4096 words
constexpr int kFlD = 512;               // model width: the dots keep their activations in registers

// Shared-memory plan (byte offsets), identical on host and device.
struct FlLayout {
  int mq, mo, m1, m2, ml;     // max rows per CTA: qkv (per cluster member), out, W1, W2, logits
  uint32_t ln_off, layer_bytes;
  uint32_t wbuf, wlog, lnf, ktile, vtile, rec, recw, slots, qkv, qkvw, xs, hs, act, red, bsm, ctl, kvstage,
      mbar, seen, svals, sidx, mt, total;
};

__host__ __device__ inline uint32_t fl_al(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline FlLayout fl_layout(int D, int F, int V, int HD, int cs, int G, int cap) {
  FlLayout Y;
  auto cr = [](int rows, int parts) { return (rows + parts - 1) / parts; };
  Y.mq = cr(3 * HD, cs);
  Y.mo = cr(D, G);
  Y.m1 = cr(F, G);
  Y.m2 = cr(D, G);
  Y.ml = cr(V, G);
  Y.ln_off = fl_al(static_cast<uint32_t>((Y.mq * D + Y.mo * D + Y.m1 * D + Y.m2 * F) * 2), 16);
  Y.layer_bytes = fl_al(Y.ln_off + 16u * D, 128);
  const int nmax = (cap + kChunk - 1) / kChunk;
  const int vec = D > F ? D : F;
  const int act = vec > V + 1 ? vec : V + 1;
  uint32_t o = 0;
  Y.wbuf = o;  o += 2 * Y.layer_bytes;
  Y.wlog = o;  o = fl_al(o + static_cast<uint32_t>(Y.ml) * D * 2, 128);
  Y.lnf = o;   o = fl_al(o + 8u * D, 128);
  Y.ktile = o; o = fl_al(o + static_cast<uint32_t>(kSlots) * kChunk * HD * 2, 128);
  Y.vtile = o; o = fl_al(o + static_cast<uint32_t>(kSlots) * kChunk * HD * 2, 128);
  Y.rec = o;   o = fl_al(o + static_cast<uint32_t>(nmax) * (HD + 4) * 4, 128);
  Y.recw = o;  o = fl_al(o + static_cast<uint32_t>(nmax) * (HD + 2) * 8, 128);  // {value, epoch} records
  Y.slots = o; o = fl_al(o + static_cast<uint32_t>(kSlots) * (kChunk + 8) * 4, 128);
  Y.qkv = o;   o = fl_al(o + 3u * HD * 4, 128);
  Y.qkvw = o;  o = fl_al(o + 2u * 3u * HD * 8, 128);  // {value, epoch} words, by layer parity
  Y.xs = o;    o = fl_al(o + 4u * D, 128);
  Y.hs = o;    o = fl_al(o + 4u * D, 128);
  Y.act = o;   o = fl_al(o + 4u * act, 128);
  Y.red = o;   o += 64 * 4;
  Y.bsm = o;   o = fl_al(o + 4u * (Y.mq + Y.mo + Y.m1 + Y.m2), 16);
  Y.ctl = o;   o += 16 * 4;
  Y.kvstage = o; o = fl_al(o + 4u * HD, 16);
  Y.mbar = o;  o += 8 * 8;
  Y.seen = o;  o = fl_al(o + V, 16);
  Y.svals = o; o = fl_al(o + 4u * V, 16);   // top-k sampling: penalised values
  Y.sidx = o;  o = fl_al(o + 4u * V, 16);   // ... and their token ids
  Y.mt = o;    o = fl_al(o + 8u * 313, 16); // mt19937_64 state + index
  Y.total = o + 128;  // alignment slack of the dynamic shared-memory base
  return Y;
}

struct FlowArgs {
  uint64_t* xattn;  // [2][D] exchange words {value bits (low), epoch (high)}
  uint64_t* xhpre;  // [2][D]
  uint64_t* xff;    // [2][F]
  uint64_t* xxpre;  // [2][D]
  uint64_t* xlog;   // [2][vp]
  int vp;           // V rounded up to even
  int cs;           // CTAs per cluster (the first H clusters each own a head)
  uint32_t epoch0;  // this launch's epochs are epoch0 + 1 ...
  uint32_t spin;    // polls of one exchange word pair before it gives up
  FlLayout y;
};

// ------------------------------------------------------------ exchange words
__device__ __forceinline__ void xw_put(uint64_t* p, float v, uint32_t ep) {
  const uint64_t w = (static_cast<uint64_t>(ep) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// After a thread's last exchange store of a phase: wait until its stores are
// performed at GPU scope, which pushes them out of the SM at once instead of
// whenever the store path drains (measured: a 132-CTA exchange round of
// 1.38 us becomes 1.06 us).
__device__ __forceinline__ void xw_flush() { __threadfence(); }
__device__ __forceinline__ void xw_get2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool xw_ready(uint64_t a, uint64_t b, uint32_t ep) {
  return static_cast<uint32_t>(a >> 32) == ep && static_cast<uint32_t>(b >> 32) == ep;
}

// Whole CTA: dst[0, n) <- the values of exchange words X[0, n) once each
// carries epoch `ep` (n even, X 16-byte aligned, n <= 2 * kThreads *
// kFlMaxPairs).  Every load of a thread is in flight at once; only the words
// not yet ready are polled again.  Returns false (for the whole CTA) when it
// gave up: this CTA had already failed (no waiting then), another CTA
// recorded a failure in the status word, or the spin budget ran out (which
// records GSVK_ERR_TIMEOUT).  Ends with a CTA barrier.
__device__ __forceinline__ bool fl_poll(const uint64_t* X, int n, uint32_t ep, float* dst,
                                        uint32_t* status, bool failed, uint32_t spin) {
  const int np = n >> 1;
  uint64_t a[kFlMaxPairs], b[kFlMaxPairs];
  bool ok = !failed;
  // no thread polls while another warp of the CTA still computes: spinning
  // warps would take issue slots and load bandwidth from it
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kFlMaxPairs; ++u) {
    a[u] = 0;
    b[u] = 0;
    const int p = threadIdx.x + u * kThreads;
    if (ok && p < np) xw_get2(X + 2 * p, a[u], b[u]);
  }
  if (ok) {
    for (uint32_t it = 0;; ++it) {
      bool all = true;
#pragma unroll
      for (int u = 0; u < kFlMaxPairs; ++u) {
        const int p = threadIdx.x + u * kThreads;
        if (p < np && !xw_ready(a[u], b[u], ep)) all = false;
      }
      if (all) break;
      if (it >= spin) {
        atomicExch(status, DEV_TIMEOUT);
        ok = false;
        break;
      }
      if ((it & 255u) == 255u && *reinterpret_cast<volatile uint32_t*>(status) != 0) {
        ok = false;
        break;
      }
#pragma unroll
      for (int u = 0; u < kFlMaxPairs; ++u) {
        const int p = threadIdx.x + u * kThreads;
        if (p < np && !xw_ready(a[u], b[u], ep)) xw_get2(X + 2 * p, a[u], b[u]);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < kFlMaxPairs; ++u) {
    const int p = threadIdx.x + u * kThreads;
    if (p < np) {
      dst[2 * p] = __uint_as_float(static_cast<uint32_t>(a[u]));
      dst[2 * p + 1] = __uint_as_float(static_cast<uint32_t>(b[u]));
    }
  }
  return __syncthreads_or(ok ? 0 : 1) == 0;
}

// W1 rows r in [a0, a1) of this CTA: relu(dot32(W1[r], x) + bias) -> xf,
// x = fp16-rounded LN1(h) formed per lane from the raw rows h.
__device__ __forceinline__ void fl_w1_rows(const uint16_t* W1, const float* h, float mean, float rstd,
                                        const float* g, const float* b, int a0, int a1, int D,
                                        const float* bias, uint64_t* xf, uint32_t ep) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a0 + 2 * warp >= a1) return;
  auto put = [&](int r, float acc) {
    const float v = __fadd_rn(acc, bias[r - a0]);
    xw_put(xf + r, v > 0.f ? v : 0.f, ep);
  };
  uint16_t xh[16];  // fp16 activations: mixed-precision fma, no conversions
  lane_act512_h(h, true, mean, rstd, g, b, xh);
  for (int r = a0 + 2 * warp; r < a1; r += 2 * kWarps) {
    if (r + 1 < a1) {
      float r0, r1;
      warp_dot512x2_h(W1 + static_cast<size_t>(r - a0) * D, W1 + static_cast<size_t>(r + 1 - a0) * D, xh,
                      &r0, &r1);
      if (lane == 0) {
        put(r, r0);
        put(r + 1, r1);
      }
    } else {
      const float r0 = warp_dot512_h(W1 + static_cast<size_t>(r - a0) * D, xh);
      if (lane == 0) put(r, r0);
    }
  }
  if (lane == 0) xw_flush();
}

// attn_combine's arithmetic with the per-record work in parallel: lane c
// holds record c's maximum and weight exp(m_c - M) (records of 32 at a time),
// then every lane runs its dimension's chain over the records in order.
// One warp; rec in shared memory; same results as attn_combine.
template <int HD>
__device__ __forceinline__ void fl_combine(const float* rec, int nch, float* out0, float* out1) {
  const int lane = threadIdx.x & 31;
  constexpr int R = rec_floats<HD>();
  float M = -INFINITY;
  for (int c0 = 0; c0 < nch; c0 += 32)
    if (c0 + lane < nch) M = fmaxf(M, rec[(c0 + lane) * R]);
  M = warp_max(M);
  float L = 0.f, O0 = 0.f, O1 = 0.f;
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const float wl = c0 + lane < nch ? exp_det(__fsub_rn(rec[(c0 + lane) * R], M)) : 0.f;
    const int n = min(32, nch - c0);
    // eight records at a time: every load and weight ahead of the chains
    for (int j0 = 0; j0 < n; j0 += 8) {
      float w[8], rl[8], r0[8], r1[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        w[u] = __shfl_sync(0xffffffffu, wl, j0 + u);
        const float* r = rec + (c0 + min(j0 + u, n - 1)) * R;  // in bounds; unused past n
        rl[u] = r[1];
        r0[u] = r[4 + lane];
        r1[u] = HD > 32 ? r[4 + 32 + lane] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u < n) {
          L = __fadd_rn(L, __fmul_rn(rl[u], w[u]));
          O0 = __fadd_rn(O0, __fmul_rn(r0[u], w[u]));
          if (HD > 32) O1 = __fadd_rn(O1, __fmul_rn(r1[u], w[u]));
        }
      }
    }
  }
  const float inv = __fdiv_rn(1.0f, L);
  *out0 = __fmul_rn(O0, inv);
  *out1 = HD > 32 ? __fmul_rn(O1, inv) : 0.f;
}

// --------------------------------------------------------------- cluster ops
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u64(uint32_t addr, uint64_t v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_volatile_shared_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.shared.u64 %0, [%1];" : "=l"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// All threads of every CTA of the cluster.  Arrive has release and wait
// acquire semantics at cluster scope: shared-memory stores into other CTAs
// before the barrier are visible to them after it.
__device__ __forceinline__ void fl_cluster_sync() {
  __syncwarp();
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// One 64-slot chunk of the canonical softmax for one head, by a slot of 64
// threads (named barrier bar_id), from K/V tiles in shared memory (row t =
// key k0 + t, HD halves per row): the arithmetic of attn_chunk_slot.  The
// record {m, l, o[HD]}, each a {value, epoch ep} word, goes to shared memory
// address `dst` (any CTA of the cluster).
template <int HD>
__device__ __forceinline__ void fl_chunk(const float* q, const uint16_t* kt, const uint16_t* vt, int nk, float scale,
                         float* ew, int bar_id, uint32_t dst, uint32_t ep) {
  float* red = ew + kChunk;
  const int t = threadIdx.x & 63, lane = t & 31, w = t >> 5;
  constexpr int kV = HD / 8;
  float qr[HD];
#pragma unroll
  for (int p = 0; p < HD / 4; ++p) {
    const float4 v = reinterpret_cast<const float4*>(q)[p];
    qr[4 * p] = v.x;
    qr[4 * p + 1] = v.y;
    qr[4 * p + 2] = v.z;
    qr[4 * p + 3] = v.w;
  }
  uint4 kr[kV];
#pragma unroll
  for (int p = 0; p < kV; ++p) kr[p] = reinterpret_cast<const uint4*>(kt + t * HD)[p];
  float score = -INFINITY;
  if (t < nk) score = __fmul_rn(thread_dot_kv<HD>(qr, kr), scale);
  float mx = warp_max(score);
  if (lane == 0) red[w] = mx;
  slot_sync(bar_id);
  mx = fmaxf(red[0], red[1]);
  ew[t] = t < nk ? exp_det(__fsub_rn(score, mx)) : 0.f;
  slot_sync(bar_id);
  // o (one dimension per lane, HD == 64: both warps) and l (warp 1 lane 0):
  // sequential sums in key order; a full chunk takes every load up front
  const int d = (HD == 64 ? 32 * w : 0) + lane;
  float o = 0.f, l = 0.f;
  if (HD == 64 || w == 0) {
    if (nk == kChunk) {
      float vv[kChunk];
#pragma unroll
      for (int k = 0; k < kChunk; ++k) vv[k] = h2f(vt[k * HD + d]);
#pragma unroll
      for (int k = 0; k < kChunk; k += 4) {
        const float4 e = reinterpret_cast<const float4*>(ew)[k / 4];
        o = __fadd_rn(o, __fmul_rn(e.x, vv[k]));
        o = __fadd_rn(o, __fmul_rn(e.y, vv[k + 1]));
        o = __fadd_rn(o, __fmul_rn(e.z, vv[k + 2]));
        o = __fadd_rn(o, __fmul_rn(e.w, vv[k + 3]));
      }
    } else {
      for (int k = 0; k < nk; ++k) o = __fadd_rn(o, __fmul_rn(ew[k], h2f(vt[k * HD + d])));
    }
  }
  if (w == 1 && lane == 0) {
    if (nk == kChunk) {
#pragma unroll
      for (int k = 0; k < kChunk; k += 4) {
        const float4 e = reinterpret_cast<const float4*>(ew)[k / 4];
        l = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(l, e.x), e.y), e.z), e.w);
      }
    } else {
      for (int k = 0; k < nk; ++k) l = __fadd_rn(l, ew[k]);
    }
  }
  const bool do_o = (HD == 64) || (w == 0);
  const bool do_l = (w == 1 && lane == 0);
  const uint64_t tag = static_cast<uint64_t>(ep) << 32;
  if (do_o) st_cluster_u64(dst + 8u * (2 + d), tag | __float_as_uint(o));
  if (do_l) {
    st_cluster_u64(dst, tag | __float_as_uint(mx));
    st_cluster_u64(dst + 8u, tag | __float_as_uint(l));
  }
  slot_sync(bar_id);
}

// ---------------------------------------------------------- top-k sampling
// std::mt19937_64 (Matsumoto-Nishimura 64-bit Mersenne Twister with the
// parameters the C++ standard fixes for it), one thread: state[0..311],
// state[312] = index of the next word.
constexpr int kMtN = 312, kMtM = 156;
__device__ void mt_seed(uint64_t* st, uint64_t seed) {
  st[0] = seed;
  for (int i = 1; i < kMtN; ++i)
    st[i] = 6364136223846793005ull * (st[i - 1] ^ (st[i - 1] >> 62)) + static_cast<uint64_t>(i);
  st[kMtN] = kMtN;
}
__device__ uint64_t mt_next(uint64_t* st) {
  if (st[kMtN] >= static_cast<uint64_t>(kMtN)) {
    constexpr uint64_t kUpper = 0xFFFFFFFF80000000ull, kLower = 0x7FFFFFFFull;
    constexpr uint64_t kA = 0xB5026F5AA96619E9ull;
    for (int i = 0; i < kMtN; ++i) {
      const uint64_t y = (st[i] & kUpper) | (st[(i + 1) % kMtN] & kLower);
      st[i] = st[(i + kMtM) % kMtN] ^ (y >> 1) ^ ((y & 1ull) ? kA : 0ull);
    }
    st[kMtN] = 0;
  }
  uint64_t x = st[st[kMtN]++];
  x ^= (x >> 29) & 0x5555555555555555ull;
  x ^= (x << 17) & 0x71D67FFFEDA60000ull;
  x ^= (x << 37) & 0xFFF7EEE000000000ull;
  x ^= x >> 43;
  return x;
}

// topk_sample (t2s_engine.cpp:1640-1737) after the penalty: vals / idx hold
// the penalised logits of tokens [0, limit) and their ids.  The top-k
// selection sort runs round by round on the whole CTA (each round the first
// position holding the maximum of positions [i, limit) -- the reference's
// strict '>' scan -- is swapped into position i); thread 0 then applies the
// temperature, the softmax (exp_det), top-p and the multinomial draw.
// Returns the token on thread 0.
__device__ int fl_topk_sample(float* vals, int* idx, int limit, int top_k, float top_p,
                              float temperature, uint64_t* mt, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = top_k > limit ? limit : (top_k < 1 ? 1 : top_k);
  for (int i = 0; i < k; ++i) {
    float bv = -INFINITY;
    int bp = 0x7fffffff;
    for (int p = i + tid; p < limit; p += kThreads) {
      const float v = vals[p];
      if (v > bv || (v == bv && p < bp)) {
        bv = v;
        bp = p;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int op = __shfl_xor_sync(0xffffffffu, bp, o);
      if (ov > bv || (ov == bv && op < bp)) {
        bv = ov;
        bp = op;
      }
    }
    if (lane == 0) {
      red[warp] = bv;
      reinterpret_cast<int*>(red + kWarps)[warp] = bp;
    }
    __syncthreads();
    if (tid == 0) {
      float B = red[0];
      int P = reinterpret_cast<int*>(red + kWarps)[0];
      for (int w = 1; w < kWarps; ++w) {
        const float ov = red[w];
        const int op = reinterpret_cast<int*>(red + kWarps)[w];
        if (ov > B || (ov == B && op < P)) {
          B = ov;
          P = op;
        }
      }
      if (vals[i] != vals[i] || P >= limit) P = i;  // a NaN at i: nothing compares greater
      if (P != i) {
        const float tv = vals[i];
        vals[i] = vals[P];
        vals[P] = tv;
        const int ti = idx[i];
        idx[i] = idx[P];
        idx[P] = ti;
      }
    }
    __syncthreads();
  }
  int tok = idx[0];
  if (tid == 0 && temperature > 0.f) {
    if (temperature != 1.0f)
      for (int i = 0; i < k; ++i) vals[i] = __fdiv_rn(vals[i], temperature);
    float mx = vals[0];
    for (int i = 1; i < k; ++i)
      if (vals[i] > mx) mx = vals[i];
    float sum = 0.f;
    for (int i = 0; i < k; ++i) {
      vals[i] = exp_det(__fsub_rn(vals[i], mx));
      sum = __fadd_rn(sum, vals[i]);
    }
    int keep = k;
    if (top_p < 1.0f) {
      const float threshold = __fmul_rn(__fsub_rn(1.f, top_p), sum);
      float cum = 0.f;
      for (int i = k - 1; i >= 0; --i) {
        cum = __fadd_rn(cum, vals[i]);
        if (cum >= threshold) {
          keep = i + 1;
          break;
        }
      }
      if (keep < k) {
        sum = 0.f;
        for (int i = 0; i < keep; ++i) sum = __fadd_rn(sum, vals[i]);
      }
    }
    // uniform_real_distribution<float>(0, 1) on the 64-bit engine (libc++
    // generate_canonical<float, 24>): one draw, as float, times 2^-64
    const float u = __fmul_rn(__fmul_rn(__ull2float_rn(mt_next(mt)), 0x1p-64f), sum);
    float cdf = 0.f;
    tok = idx[keep - 1];
    for (int i = 0; i < keep; ++i) {
      cdf = __fadd_rn(cdf, vals[i]);
      if (u <= cdf) {
        tok = idx[i];
        break;
      }
    }
  }
  return tok;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    t2s_flow_kernel(const T2SDev m, const DecodeArgs a, const FlowArgs f,
                    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<128>(smem_raw);
  const FlLayout& Y = f.y;
  const int D = m.D, F = m.F, V = m.V, L = m.L, cap = m.cap;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x, cs = f.cs;
  const int head = c / cs;
  // clusters past the heads help with the grid-wide rows only (no q/k/v rows,
  // no attention): the GPU holds fewer clusters of a given size than it has
  // SMs for, so the grid is H head clusters plus as many helpers as fit
  const bool is_head = head < m.H;
  const int rank = static_cast<int>(cluster_rank());

  uint8_t* const wbuf0 = smem + Y.wbuf;  // layer buffer b at wbuf0 + b * layer_bytes
  uint16_t* wlog = reinterpret_cast<uint16_t*>(smem + Y.wlog);
  float* lnf = reinterpret_cast<float*>(smem + Y.lnf);
  uint16_t* ktile = reinterpret_cast<uint16_t*>(smem + Y.ktile);
  uint16_t* vtile = reinterpret_cast<uint16_t*>(smem + Y.vtile);
  float* rec = reinterpret_cast<float*>(smem + Y.rec);
  uint64_t* recw = reinterpret_cast<uint64_t*>(smem + Y.recw);
  float* slots = reinterpret_cast<float*>(smem + Y.slots);
  float* qkv = reinterpret_cast<float*>(smem + Y.qkv);
  uint64_t* qkvw = reinterpret_cast<uint64_t*>(smem + Y.qkvw);
  float* xs = reinterpret_cast<float*>(smem + Y.xs);
  float* hs = reinterpret_cast<float*>(smem + Y.hs);
  float* act = reinterpret_cast<float*>(smem + Y.act);
  float* red = reinterpret_cast<float*>(smem + Y.red);
  float* bsm = reinterpret_cast<float*>(smem + Y.bsm);
  int* ctl = reinterpret_cast<int*>(smem + Y.ctl);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + Y.mbar);
  uint8_t* seen = smem + Y.seen;
  float* svals = reinterpret_cast<float*>(smem + Y.svals);
  int* sidx = reinterpret_cast<int*>(smem + Y.sidx);
  uint64_t* mt = reinterpret_cast<uint64_t*>(smem + Y.mt);
  const bool topk = a.samp_mode == 1;
  const float pen = topk ? a.samp_pen : 1.35f;

  // row ownership: qkv rows of this cluster's head (local index j: group
  // j / HD = q, k, v; element j % HD), the other matrices over the grid
  const int j0 = is_head ? row_lo(3 * HD, cs, rank) : 0;
  const int j1 = is_head ? row_lo(3 * HD, cs, rank + 1) : 0;
  const int o0 = row_lo(D, G, c), o1 = row_lo(D, G, c + 1);
  const int a0 = row_lo(F, G, c), a1 = row_lo(F, G, c + 1);
  const int b0 = row_lo(D, G, c), b1 = row_lo(D, G, c + 1);
  const int l0 = row_lo(V, G, c), l1 = row_lo(V, G, c + 1);
  const int nq = j1 - j0, no = o1 - o0, na = a1 - a0, nb = b1 - b0;
  auto qkv_row = [&](int j) { return (j / HD) * D + head * HD + (j % HD); };
  // The bias this thread stages for layer l: the address is chosen first and
  // loaded once (a select between loaded values would wait for the loads).
  // Threads without a row load any valid word; bsm ignores it.
  auto bias_of = [&](int l) -> float {
    const size_t L_ = static_cast<size_t>(l);
    const float* p = m.bout;
    if (tid < nq)
      p = m.bqkv + L_ * 3 * D + qkv_row(j0 + tid);
    else if (tid < nq + no)
      p = m.bout + L_ * D + o0 + tid - nq;
    else if (tid < nq + no + na)
      p = m.b1 + L_ * F + a0 + tid - nq - no;
    else if (tid < nq + no + na + nb)
      p = m.b2 + L_ * D + b0 + tid - nq - no - na;
    return __ldg(p);
  };
  // Part `part` (0..4) of layer l's weight slices into buffer `buf`; part 0
  // posts the whole layer's byte count.
  auto prefetch = [&](int l, uint8_t* buf, uint64_t* bar, int part) {
    const size_t Dz = D, Fz = F;
    uint8_t* pq = buf;
    uint8_t* po = pq + static_cast<size_t>(Y.mq) * Dz * 2;
    uint8_t* p1 = po + static_cast<size_t>(Y.mo) * Dz * 2;
    uint8_t* p2 = p1 + static_cast<size_t>(Y.m1) * Dz * 2;
    const uint32_t vb = static_cast<uint32_t>(Dz) * 4;
    switch (part) {
      case 0: {
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>((nq + no + na) * Dz * 2 + nb * Fz * 2) +
                                       (l > 0 ? 4 * vb : 2 * vb));
        // the cluster's q, k and v rows of this member: up to three runs
        for (int g = 0; g < 3; ++g) {
          const int s0 = max(j0, g * HD), s1 = min(j1, (g + 1) * HD);
          if (s1 > s0)
            bulk_load(pq + static_cast<size_t>(s0 - j0) * Dz * 2,
                      m.wqkv + (static_cast<size_t>(l) * 3 * Dz + qkv_row(s0)) * Dz,
                      static_cast<uint32_t>((s1 - s0) * Dz * 2), bar);
        }
        break;
      }
      case 1:
        if (no) bulk_load(po, m.wout + (static_cast<size_t>(l) * Dz + o0) * Dz, no * Dz * 2, bar);
        break;
      case 2:
        if (na) bulk_load(p1, m.w1 + (static_cast<size_t>(l) * Fz + a0) * Dz, na * Dz * 2, bar);
        break;
      case 3: {
        const uint16_t* w2 = m.w2p ? m.w2p : m.w2;
        if (nb) bulk_load(p2, w2 + (static_cast<size_t>(l) * Dz + b0) * Fz, nb * Fz * 2, bar);
        break;
      }
      default: {
        float* ln = reinterpret_cast<float*>(buf + Y.ln_off);
        bulk_load(ln, m.n1g + static_cast<size_t>(l) * Dz, vb, bar);
        bulk_load(ln + Dz, m.n1b + static_cast<size_t>(l) * Dz, vb, bar);
        if (l > 0) {
          bulk_load(ln + 2 * Dz, m.n2g + static_cast<size_t>(l - 1) * Dz, vb, bar);
          bulk_load(ln + 3 * Dz, m.n2b + static_cast<size_t>(l - 1) * Dz, vb, bar);
        }
      }
    }
  };
  // Chunks of this member in attention round rd over nch chunks: slot s
  // takes chunk (rd * kSlots + s) * cs + rank.
  auto chunk_of = [&](int rd, int s) { return (rd * kSlots + s) * cs + rank; };
  // Thread 0: TMA loads of this member's K/V tiles of layer l, round rd, for
  // a pass over nch chunks.  Returns whether anything was issued (then the
  // tile barrier completes once).
  auto issue_tiles = [&](int l, int nch, int rd) -> bool {
    uint32_t bytes = 0;
    for (int s = 0; s < kSlots; ++s)
      if (chunk_of(rd, s) < nch) bytes += 2u * kChunk * HD * 2;
    if (!bytes) return false;
    mbar_arrive_expect_tx(&mbar[3], bytes);
    for (int s = 0; s < kSlots; ++s) {
      const int ch = chunk_of(rd, s);
      if (ch >= nch) continue;
      tma_load_2d(ktile + s * kChunk * HD, &tmk, &mbar[3], head * HD, l * cap + ch * kChunk);
      tma_load_2d(vtile + s * kChunk * HD, &tmv, &mbar[3], head * HD, l * cap + ch * kChunk);
    }
    return true;
  };
  auto tiles_issued = [&](int nch, int rd) {
    for (int s = 0; s < kSlots; ++s)
      if (chunk_of(rd, s) < nch) return true;
    return false;
  };

  const int eos = V - 1;
  bool failed = false;
  // per layer buffer b: bit b of `phase` = parity of its next completion,
  // bit b of `pending` = a refill is in flight
  uint32_t phase = 0, pending = 3u;
  uint32_t tile_uses = 0;
  bool tiles_armed;
  {
    const int nch0 = (a.pos0 + 1 + kChunk - 1) / kChunk;
    tiles_armed = is_head && tiles_issued(nch0, 0);
  }

  for (int cc = tid; cc < V; cc += kThreads) seen[cc] = 0;
  for (int i = tid; i < 2 * 3 * HD; i += kThreads) qkvw[i] = 0;  // epoch 0 is never used
  for (int i = tid; i < (cap + kChunk - 1) / kChunk * (HD + 2); i += kThreads) recw[i] = 0;
  __syncthreads();
  for (int i = tid; i < a.n_hist; i += kThreads) {
    const int t = a.hist[i];
    if (t >= 0 && t < V) seen[t] = 1;
  }
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&mbar[i], 1);
    fence_barrier_init();
    if (topk) mt_seed(mt, a.samp_seed);  // t2s_engine.cpp:1814-1818, one engine per generate
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bl = static_cast<uint32_t>((l1 - l0) * D * 2);
    mbar_arrive_expect_tx(&mbar[2], bl + 2u * D * 4);
    if (bl) bulk_load(wlog, m.wpred + static_cast<size_t>(l0) * D, bl, &mbar[2]);
    bulk_load(lnf, m.n2g + static_cast<size_t>(L - 1) * D, D * 4, &mbar[2]);
    bulk_load(lnf + D, m.n2b + static_cast<size_t>(L - 1) * D, D * 4, &mbar[2]);
    for (int part = 0; part < 5; ++part) prefetch(0, wbuf0, &mbar[0], part);
    for (int part = 0; part < 5; ++part) prefetch(1 % L, wbuf0 + Y.layer_bytes, &mbar[1], part);
    if (is_head) issue_tiles(0, (a.pos0 + 1 + kChunk - 1) / kChunk, 0);
  }
  // every member of the cluster is running before any distributed
  // shared-memory store
  fl_cluster_sync();
  bool logits_pending = true;
  if (mbar_wait(&mbar[2], 0, m.status))
    logits_pending = false;
  else
    failed = true;
  failed = __syncthreads_or(failed ? 1 : 0) != 0;

  const uint32_t rec_remote = cluster_addr(recw, 0);  // the merger's chunk record words
  unsigned gl = 0;
  int n_out = 0;
  unsigned long long* tr = nullptr;
#define GSVK_FTR(slot)                              \
  do {                                              \
    if (tr && tid == 0) tr[(slot)] = global_ns();   \
  } while (0)
  for (int idx = 0; idx < a.max_steps; ++idx) {
    tr = (a.trace && c == 0 && idx < kTraceSteps) ? a.trace + idx * kTraceStride : nullptr;
    GSVK_FTR(0);
    const uint32_t ep_step = f.epoch0 + static_cast<uint32_t>(idx) * static_cast<uint32_t>(L + 1);
    float bias_next = bias_of(0);
    // -------------------------------------------- logits of the last step
    const float* lg = m.logits;  // step 0: the prompt's logits (an earlier launch)
    if (idx > 0) {
      const uint32_t ep = ep_step;  // the previous step's logits epoch
      if (!fl_poll(f.xlog + static_cast<size_t>(ep & 1u) * f.vp, f.vp, ep, act, m.status, failed, f.spin))
        failed = true;
      lg = act;
    }
    // -------------------------------------- greedy sample (every CTA)
    // t2s_engine.cpp:1594-1636: penalty once per distinct history token,
    // EOS excluded while idx < 11, first maximum wins.
    const int eos_allowed = idx >= 11;
    const int limit = eos_allowed ? V : V - 1;
    float bv = -INFINITY, sv = -INFINITY;
    int bi = 0x7fffffff;
    for (int cc = tid; cc < limit; cc += kThreads) {
      float v = idx > 0 ? lg[cc] : __ldcg(lg + cc);
      if (seen[cc]) v = v < 0.f ? __fmul_rn(v, pen) : __fdiv_rn(v, pen);
      if (topk) {
        svals[cc] = v;
        sidx[cc] = cc;
      }
      if (v > bv || (v == bv && cc < bi)) {
        sv = bv;
        bv = v;
        bi = cc;
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
    // top-k sampling replaces the argmax (the margins below stay top1 - top2)
    const int sampled = topk ? fl_topk_sample(svals, sidx, limit, a.samp_top_k, a.samp_top_p,
                                              a.samp_temp, mt, red + 3 * kWarps)
                             : 0;
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
      if (c == 0 && a.margins) a.margins[idx] = __fsub_rn(B, S);
      if (topk) I = sampled;
      // the cluster follows its first member's token and abort decision
      if (rank == 0) {
        const int abort = failed || I < 0 || I >= V ||
                          *reinterpret_cast<volatile uint32_t*>(m.status) != 0;
        for (int r = 0; r < cs; ++r) {
          st_cluster_u32(cluster_addr(ctl, r), static_cast<uint32_t>(I));
          st_cluster_u32(cluster_addr(ctl + 1, r), static_cast<uint32_t>(abort));
        }
      }
    }
    fl_cluster_sync();
    const int tok = ctl[0];
    const bool abort = ctl[1] != 0;
    bool stop = abort;
    if (!abort) {
      if (a.stop_on_eos && eos_allowed && tok == eos) {
        stop = true;
      } else {
        if (c == 0 && tid == 0) a.tokens[n_out] = tok;
        ++n_out;
        if (tid == 0) seen[tok] = 1;
      }
      if (idx + 1 == a.max_steps) stop = true;
    }
    __syncthreads();
    GSVK_FTR(1);
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
    const int rounds = (nch + kSlots * cs - 1) / (kSlots * cs);
    // layer 0's tiles (the first step's were issued before the loop): after
    // the step's cluster barrier, which orders every K/V row the previous
    // step stored before these loads
    if (is_head && !failed && !tiles_armed) {
      if (tid == 0) issue_tiles(0, nch, 0);
      tiles_armed = tiles_issued(nch, 0);
    }

    for (int l = 0; l < L; ++l, ++gl) {
      const uint32_t ep = ep_step + 1 + static_cast<uint32_t>(l);
      const uint32_t par = ep & 1u;
      const int b = static_cast<int>(gl & 1u);
      uint8_t* const wb = wbuf0 + static_cast<size_t>(b) * Y.layer_bytes;
      const uint16_t* Wq = reinterpret_cast<const uint16_t*>(wb);
      const uint16_t* Wo = Wq + static_cast<size_t>(Y.mq) * D;
      const uint16_t* W1 = Wo + static_cast<size_t>(Y.mo) * D;
      const uint16_t* W2 = W1 + static_cast<size_t>(Y.m1) * D;
      const float* lnb = reinterpret_cast<const float*>(wb + Y.ln_off);
      // ---------------------------------------------- layer input, QKV rows
      // a copy that was not waited for (after a failure) stays pending: the
      // exit drain waits for it, so no bulk copy outlives the CTA
      if (!failed) {
        if (mbar_wait(&mbar[b], (phase >> b) & 1u, m.status)) {
          phase ^= 1u << b;
          pending &= ~(1u << b);
        } else {
          failed = true;
        }
      }
      if (tid < nq + no + na + nb) bsm[tid] = bias_next;
      if (l > 0) {
        GSVK_FTR(16 + 16 * l + 14);
        if (!fl_poll(f.xxpre + static_cast<size_t>((ep - 1) & 1u) * D, D, ep - 1, xs, m.status,
                     failed, f.spin))
          failed = true;
        GSVK_FTR(16 + 16 * l + 15);
      }
      failed = __syncthreads_or(failed ? 1 : 0) != 0;  // one decision for the whole CTA
      // LN2 of layer l - 1 (layer 0 takes its input as it is): warp 0 forms
      // the statistics (one warp's chain loads instead of eight warps'
      // competing for shared memory), the CTA reads them after one barrier,
      // and every lane normalises only the elements its dots read, so xs
      // keeps the raw rows
      const bool ln2 = l > 0;
      float mu2 = 0.f, rs2 = 0.f;
      if (ln2) {  // warp 0 forms the statistics, the CTA reads them
        if (warp == 0) {
          warp_ln_stats(xs, kFlD, m.eps, &mu2, &rs2);
          if (lane == 0) {
            red[48] = mu2;
            red[49] = rs2;
          }
        }
        __syncthreads();
        mu2 = red[48];
        rs2 = red[49];
      }
      GSVK_FTR(16 + 16 * l + 10);
      {
        auto put = [&](int j, float acc) {
          // every lane holds acc; lanes 0..cs-1 push it to one member each
          // (k and v as their fp16 cache values)
          const float v = __fadd_rn(acc, bsm[j - j0]);
          const float val = j < HD ? v : h2f(f2h(v));
          if (lane < cs)
            st_cluster_u64(cluster_addr(qkvw + par * 3 * HD + j, lane),
                           (static_cast<uint64_t>(ep) << 32) | __float_as_uint(val));
        };
        uint16_t xh[16];  // fp16 activations (the reference's fp16 x)
        lane_act512_h(xs, ln2, mu2, rs2, lnb + 2 * D, lnb + 3 * D, xh);
        for (int j = j0 + 2 * warp; j < j1; j += 2 * kWarps) {
          if (j + 1 < j1) {
            float r0, r1;
            warp_dot512x2_h(Wq + static_cast<size_t>(j - j0) * D, Wq + static_cast<size_t>(j + 1 - j0) * D,
                            xh, &r0, &r1);
            put(j, r0);
            put(j + 1, r1);
          } else {
            put(j, warp_dot512_h(Wq + static_cast<size_t>(j - j0) * D, xh));
          }
        }
      }
      GSVK_FTR(16 + 16 * l + 0);
      // this head's q, k and v from every member: each word carries this
      // layer's epoch, so the CTA polls its own shared memory (no cluster
      // barrier) and keeps a plain copy for the chunks
      if (is_head) {
        if (tid < 3 * HD && !failed) {
          const uint64_t* w = qkvw + par * 3 * HD + tid;
          uint64_t v = ld_volatile_shared_u64(w);
          for (uint32_t it = 0; static_cast<uint32_t>(v >> 32) != ep; ++it) {
            if (it >= f.spin) {
              atomicExch(m.status, DEV_TIMEOUT);
              failed = true;
              break;
            }
            if ((it & 255u) == 255u && *reinterpret_cast<volatile uint32_t*>(m.status) != 0) {
              failed = true;
              break;
            }
            v = ld_volatile_shared_u64(w);
          }
          qkv[tid] = __uint_as_float(static_cast<uint32_t>(v));
        }
        failed = __syncthreads_or(failed ? 1 : 0) != 0;
      }
      GSVK_FTR(16 + 16 * l + 1);
      if (is_head && rank == cs - 1 && warp == kWarps - 1) {
        // the head's new K and V rows (fp16) into the cache by bulk copy (the
        // same async proxy as the TMA tile loads that read them later), by
        // the member and warp with the least attention work
        uint16_t* stg = reinterpret_cast<uint16_t*>(smem + Y.kvstage);
        for (int e = lane; e < HD; e += 32) {
          stg[e] = f2h(qkv[HD + e]);
          stg[HD + e] = f2h(qkv[2 * HD + e]);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          const size_t row = (static_cast<size_t>(l) * cap + pos) * D + head * HD;
          bulk_store(m.kc + row, stg, HD * 2);
          bulk_store(m.vc + row, stg + HD, HD * 2);
          bulk_commit();
        }
      }
      if (l + 1 < L) bias_next = bias_of(l + 1);  // the next layer's, a phase ahead
      // ------------------------------------------- attention of this head
      {
        const int slot = tid >> 6;
        float* ew = slots + slot * (kChunk + 8);
        for (int rd = 0; rd < (is_head ? rounds : 0); ++rd) {
          if (rd > 0 && !failed && !tiles_armed) {  // later rounds: refill the tiles
            __syncthreads();                           // (all slots are done with them)
            if (tid == 0) issue_tiles(l, nch, rd);
            tiles_armed = tiles_issued(nch, rd);
          }
          // tiles_armed: a tile copy in flight; one that was not waited for
          // (after a failure) stays armed for the exit drain
          if (tiles_armed && !failed) {
            if (mbar_wait(&mbar[3], tile_uses & 1u, m.status)) {
              ++tile_uses;
              tiles_armed = false;
            } else {
              failed = true;
            }
          }
          failed = __syncthreads_or(failed ? 1 : 0) != 0;
          if (rd == 0) GSVK_FTR(16 + 16 * l + 11);
          const int ch = chunk_of(rd, slot);
          if (ch < nch) {
            uint16_t* kt = ktile + slot * kChunk * HD;
            uint16_t* vt = vtile + slot * kChunk * HD;
            const int k0 = ch * kChunk;
            const int t = tid & 63;
            if (pos >= k0 && pos < k0 + kChunk && t < HD) {  // the new key: this step's k, v
              kt[(pos - k0) * HD + t] = f2h(qkv[HD + t]);
              vt[(pos - k0) * HD + t] = f2h(qkv[2 * HD + t]);
              fence_proxy_async_shared();  // before a later TMA load rewrites the tile
            }
            slot_sync(1 + slot);
            fl_chunk<HD>(qkv, kt, vt, min(len - k0, kChunk), m.scale, ew, 1 + slot,
                         rec_remote + static_cast<uint32_t>(ch) * (HD + 2) * 8u, ep);
          }
        }
      }
      GSVK_FTR(16 + 16 * l + 2);
      // the K/V row is in the cache before the next step's cluster barrier,
      // after which the tiles that read it are issued
      if (is_head && rank == cs - 1 && tid == kThreads - 32) bulk_wait<0>();
      if (is_head) {
        if (rank == 0) {
          // every member's chunk records ({value, epoch} words in this CTA's
          // shared memory), polled locally instead of a cluster barrier
          constexpr int RW = HD + 2, R = rec_floats<HD>();
          for (int i = tid; i < nch * RW && !failed; i += kThreads) {
            const uint64_t* w = recw + i;
            uint64_t v = ld_volatile_shared_u64(w);
            for (uint32_t it = 0; static_cast<uint32_t>(v >> 32) != ep; ++it) {
              if (it >= f.spin) {
                atomicExch(m.status, DEV_TIMEOUT);
                failed = true;
                break;
              }
              if ((it & 255u) == 255u && *reinterpret_cast<volatile uint32_t*>(m.status) != 0) {
                failed = true;
                break;
              }
              v = ld_volatile_shared_u64(w);
            }
            const int cr = i / RW, k = i - cr * RW;
            rec[cr * R + (k < 2 ? k : k + 2)] = __uint_as_float(static_cast<uint32_t>(v));
          }
          failed = __syncthreads_or(failed ? 1 : 0) != 0;
          GSVK_FTR(16 + 16 * l + 3);
          if (warp == 0) {  // merge the head's chunk records, canonical order
            float r0, r1;
            fl_combine<HD>(rec, nch, &r0, &r1);
            uint64_t* xa = f.xattn + static_cast<size_t>(par) * D + head * HD;
            xw_put(xa + lane, h2f(f2h(r0)), ep);
            if (HD > 32) xw_put(xa + 32 + lane, h2f(f2h(r1)), ep);
            xw_flush();
          }
        } else {
          __syncthreads();  // every slot is done with the tiles before they are refilled
        }
        // the next layer's tiles (the next step's first layer: after that
        // step's cluster barrier)
        if (l + 1 < L && !failed && !tiles_armed) {
          if (tid == 0) issue_tiles(l + 1, nch, 0);
          tiles_armed = tiles_issued(nch, 0);
        }
      }
      GSVK_FTR(16 + 16 * l + 13);
      // ------------------------------------------------ out-proj rows
      if (!fl_poll(f.xattn + static_cast<size_t>(par) * D, D, ep, act, m.status, failed, f.spin)) failed = true;
      GSVK_FTR(16 + 16 * l + 4);
      if (o0 + warp < o1) {
        uint16_t xh[16];  // the attention output: fp16 values, exact as fp16 bits
        lane_act512_h(act, false, 0.f, 0.f, nullptr, nullptr, xh);
        for (int r = o0 + warp; r < o1; r += kWarps) {
          const float acc = warp_dot512_h(Wo + static_cast<size_t>(r - o0) * D, xh);
          if (lane == 0) {
            // the residual: this layer's input row (LN2 output of layer l - 1)
            const float xin = ln2 ? ln_val(xs[r], mu2, rs2, lnb[2 * D + r], lnb[3 * D + r]) : xs[r];
            xw_put(f.xhpre + static_cast<size_t>(par) * D + r, __fadd_rn(__fadd_rn(acc, bsm[nq + r - o0]), xin),
                   ep);
          }
        }
        if (lane == 0) xw_flush();
      }
      // ------------------------------------------- LN1, W1 rows + ReLU
      if (!fl_poll(f.xhpre + static_cast<size_t>(par) * D, D, ep, hs, m.status, failed, f.spin)) failed = true;
      GSVK_FTR(16 + 16 * l + 5);
      // LN1 as LN2 above: hs keeps the raw rows
      float mu1, rs1;
      if (warp == 0) {
        warp_ln_stats(hs, kFlD, m.eps, &mu1, &rs1);
        if (lane == 0) {
          red[50] = mu1;
          red[51] = rs1;
        }
      }
      __syncthreads();
      mu1 = red[50];
      rs1 = red[51];
      GSVK_FTR(16 + 16 * l + 12);
      fl_w1_rows(W1, hs, mu1, rs1, lnb, lnb + D, a0, a1, D, bsm + nq + no, f.xff + static_cast<size_t>(par) * F,
                 ep);
      GSVK_FTR(16 + 16 * l + 6);
      // ------------------------------------------------------- W2 rows
      if (!fl_poll(f.xff + static_cast<size_t>(par) * F, F, ep, act, m.status, failed, f.spin)) failed = true;
      GSVK_FTR(16 + 16 * l + 7);
      {
        uint64_t* xx = f.xxpre + static_cast<size_t>(par) * D;
        if (m.w2p) {  // lane-ordered W2 slice (F = kClF), activations in registers
          float xr[2 * kClFB];
          lane_load_x(act, xr);
          for (int r = b0 + warp; r < b1; r += kWarps) {
            const float acc = lane_dot_ordered(W2 + static_cast<size_t>(r - b0) * F, xr);
            if (lane == 0)
              xw_put(xx + r, __fadd_rn(__fadd_rn(acc, bsm[nq + no + na + r - b0]),
                                       ln_val(hs[r], mu1, rs1, lnb[r], lnb[D + r])), ep);
          }
          if (lane == 0 && b0 + warp < b1) xw_flush();
        } else {
          for (int r = b0 + warp; r < b1; r += kWarps) {
            const float acc = warp_dot32(W2 + static_cast<size_t>(r - b0) * F, act, F);
            if (lane == 0)
              xw_put(xx + r, __fadd_rn(__fadd_rn(acc, bsm[nq + no + na + r - b0]),
                                       ln_val(hs[r], mu1, rs1, lnb[r], lnb[D + r])), ep);
          }
          if (lane == 0 && b0 + warp < b1) xw_flush();
        }
      }
      GSVK_FTR(16 + 16 * l + 8);
      // every warp is done with wbuf[b]: refill it with global layer gl + 2
      __syncthreads();
      if (!failed) {
        if (lane == 0 && warp >= 1 && warp <= 5) prefetch((l + 2) % L, wb, &mbar[b], warp - 1);
        pending |= 1u << b;
      }
      GSVK_FTR(16 + 16 * l + 9);
    }
    // ---------------------------------------------------------------- logits
    {
      const uint32_t ep_x = ep_step + static_cast<uint32_t>(L);  // layer L - 1
      const uint32_t ep_l = ep_step + static_cast<uint32_t>(L) + 1;
      if (!fl_poll(f.xxpre + static_cast<size_t>(ep_x & 1u) * D, D, ep_x, xs, m.status, failed, f.spin))
        failed = true;
      // the final LayerNorm per warp, fp32 activations
      float muf, rsf, xr[16];
      warp_ln_stats(xs, kFlD, m.eps, &muf, &rsf);
      lane_act512(xs, true, muf, rsf, lnf, lnf + D, false, xr);
      uint64_t* xl = f.xlog + static_cast<size_t>(ep_l & 1u) * f.vp;
      for (int r = l0 + warp; r < l1; r += kWarps) {
        const float acc = warp_dot512_r(wlog + static_cast<size_t>(r - l0) * D, xr);
        if (lane == 0) {
          xw_put(xl + r, acc, ep_l);
          m.logits[r] = acc;
          if (r == V - 1 && f.vp > V) xw_put(xl + V, 0.f, ep_l);  // the padding word
        }
      }
      if (lane == 0 && l0 + warp < l1) xw_flush();
      GSVK_FTR(2);
    }
  }
#undef GSVK_FTR
  // Leave together (no member exits while another may still store into its
  // shared memory), then drain bulk copies still in flight.
  fl_cluster_sync();
  if (tid == 0) {
    for (int bb = 0; bb < 2; ++bb)
      if ((pending >> bb) & 1u) mbar_wait(&mbar[bb], (phase >> bb) & 1u, m.status);
    if (tiles_armed) mbar_wait(&mbar[3], tile_uses & 1u, m.status);
    if (logits_pending) mbar_wait(&mbar[2], 0, m.status);
    if (c == 0 && a.n_out) *a.n_out = n_out;
  }
  bulk_wait<0>();  // the K/V row stores of the thread that issued them
  __syncthreads();
}
