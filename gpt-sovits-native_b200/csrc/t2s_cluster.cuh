// t2s_cluster.cuh — batch-1 T2S decode on ONE thread-block cluster.
// Included by t2s.cu inside its anonymous namespace (it shares T2SDev,
// DecodeArgs, the attention slot helpers and the canonical arithmetic).
//
// The grid-wide t2s_decode_kernel synchronises 148 CTAs 121 times per token,
// and a grid barrier costs ~1.2 us on this part.  Here the whole generation
// runs on one cluster of kClCS CTAs (16, a non-portable cluster size), where
// the hardware cluster barrier costs ~0.25 us and results move through
// distributed shared memory:
//   * each CTA streams its row slices of every weight matrix, layer after
//     layer and step after step, through a ring of kClRing bulk-copy slots:
//     after all warps are done with chunk c, thread 0 refills its slot with
//     chunk c + kClRing (so the copies run kClRing - 1 chunks ahead);
//   * the phases P1..P5 of t2s_decode_kernel run with the same canonical
//     arithmetic, and each phase's outputs are pushed into every CTA's copy
//     of the vector (stores through mapa'd addresses) before the barrier;
//   * control flow is identical in every CTA (the stop decision comes from
//     the pushed logits, which every CTA holds identically), so every CTA
//     passes the same sequence of cluster barriers; a bounded wait that
//     gives up records GSVK_ERR_TIMEOUT and stops waiting from then on.
// Dot products of 512-wide rows use an 8-threads-per-row layout: thread g of
// a row runs the four accumulator chains that lanes 4g..4g+3 run in
// warp_dot32 (same products, same order, same final association), with its
// activations in registers; 2048-wide rows keep warp_dot32's lane layout,
// again with the activations in registers.  Results are bit-identical to
// t2s_decode_kernel.

constexpr int kClCS = 16;                    // CTAs in the cluster
constexpr int kClWarps = 12;                 // warps per CTA
constexpr int kClCons = kClWarps * 32;       // 384 threads
constexpr int kClThreads = kClCons;
constexpr int kClSlots = kClCons / 64;       // attention slots (64 threads each)
constexpr int kClRing = 3;                   // weight ring depth
constexpr uint32_t kClSlotBytes = 48u * 1024u;
constexpr int kClMaxChunks = 64;             // key chunks per head (cap <= 4096)
constexpr int kClD = 512, kClF = 2048, kClHD = 32;
constexpr int kClNB = kClD / 64;             // 64-element blocks of a D row
constexpr int kClFB = kClF / 64;             // ... of an F row
constexpr int kClStg = 128;                  // staged outputs per CTA and phase (max slice)
constexpr int kClBias = 96 + 32 + 128 + 32;  // bias slices of one layer (qkv, out, w1, w2)

// Dynamic shared memory plan (floats after the ring), identical on host and device.
struct ClLayout {
  uint32_t xin, qv, att, hp, ffv, x16, att16, hp16, bsm, stg, slots, rec, red, seen, total;
};
__host__ __device__ inline ClLayout cl_layout(int V) {
  ClLayout L;
  uint32_t f = kClRing * kClSlotBytes / 4;
  L.xin = f;   f += kClD;
  L.qv = f;    f += kClD;
  L.att = f;   f += kClD;
  L.hp = f;    f += kClD;
  L.ffv = f;   f += (V > kClF ? V : kClF);         // also the pushed logits
  f = (f + 3) & ~3u;
  L.x16 = f;   f += kClD / 2;                      // fp16 copies of xin, att, hp
  L.att16 = f; f += kClD / 2;
  L.hp16 = f;  f += kClD / 2;
  L.bsm = f;   f += kClBias;
  L.stg = f;   f += kClStg;
  L.slots = f; f += kClSlots * slot_floats<kClHD>();
  L.rec = f;   f += kClMaxChunks * rec_floats<kClHD>();
  L.red = f;   f += 64;
  L.seen = f;  f += (V + 3) / 4;
  L.total = f * 4;
  return L;
}

__device__ __forceinline__ void cons_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kClCons) : "memory");
}
__device__ __forceinline__ uint32_t cl_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Generic address of the same shared-memory object in CTA `rank` of the cluster.
template <typename T>
__device__ __forceinline__ T* cl_map(T* p, uint32_t rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
  return reinterpret_cast<T*>(r);
}
// Hardware cluster barrier (arrive: release, wait: acquire, cluster scope).
__device__ __forceinline__ void cl_barrier_all() {
  __syncwarp();  // .aligned: the whole warp executes it together
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
// Wait for a ring slot's copy.  One lane per warp polls (no suspend hint);
// the other lanes park at the warp barrier so that they take no issue slots
// from warps still computing; then every lane confirms the phase itself (an
// immediate success that gives it acquire ordering on the copied data).
// Bounded: after one timeout the kernel no longer waits, so a failed launch
// still runs to its end and reports the status.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Warp-collective: every lane of the warp must call it together.
__device__ __forceinline__ void cl_wait_full(uint64_t* bar, uint32_t parity, uint32_t* status,
                                             bool& failed) {
  if (failed) return;
  bool ok = true;
  if ((threadIdx.x & 31) == 0) {
    ok = false;
    for (uint32_t i = 0; i < kSpinLimit && !ok; ++i) ok = mbar_test(bar, parity);
    if (!ok) atomicExch(status, DEV_TIMEOUT);
  }
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (!ok) {
    failed = true;
    return;
  }
  mbar_test(bar, parity);
}

// ln_canon (kern.cpp:27-58 order) for the 384 threads: thread t holds the
// LayerNorm parameters of elements t and t + kClCons in registers.
__device__ void ln_cons(float* buf, int n, double eps, float* scratch, float gA, float bA, float gB,
                        float bB, uint16_t* out16) {
  const int tid = threadIdx.x;
  const int vec_end = n & ~7;
  if (tid < 16) {
    const int l = tid & 7;
    const bool sq = tid >= 8;
    float a = 0.f;
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
    scratch[tid] = a;
  }
  cons_sync();
  if (tid == 0) {
    const float* f = scratch;
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(f[0], f[1]), __fadd_rn(f[2], f[3])),
                              __fadd_rn(__fadd_rn(f[4], f[5]), __fadd_rn(f[6], f[7])));
    const float q = __fadd_rn(__fadd_rn(__fadd_rn(f[8], f[9]), __fadd_rn(f[10], f[11])),
                              __fadd_rn(__fadd_rn(f[12], f[13]), __fadd_rn(f[14], f[15])));
    double sum = static_cast<double>(s), sqs = static_cast<double>(q);
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
    const float rstd = static_cast<float>(
        __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(static_cast<double>(var), eps))));
    scratch[16] = mean;
    scratch[17] = rstd;
  }
  cons_sync();
  const float mean = scratch[16], rstd = scratch[17];
  if (tid < n) {
    const float v = fmaf(__fmul_rn(__fsub_rn(buf[tid], mean), rstd), gA, bA);
    buf[tid] = v;
    if (out16) out16[tid] = f2h(v);
  }
  if (tid + kClCons < n) {
    const float v = fmaf(__fmul_rn(__fsub_rn(buf[tid + kClCons], mean), rstd), gB, bB);
    buf[tid + kClCons] = v;
    if (out16) out16[tid + kClCons] = f2h(v);
  }
  cons_sync();
}

// Activations of a 512-wide row for the 8-threads-per-row layout:
// xr[8b + u] = x[64b + 8g + u], g = thread & 7 (optionally rounded to fp16).
__device__ __forceinline__ void g8_load_x(const float* x, float* xr, bool round16) {
  const int g = threadIdx.x & 7;
#pragma unroll
  for (int b = 0; b < kClNB; ++b) {
    const float4 lo = *reinterpret_cast<const float4*>(x + 64 * b + 8 * g);
    const float4 hi = *reinterpret_cast<const float4*>(x + 64 * b + 8 * g + 4);
    xr[8 * b] = lo.x;
    xr[8 * b + 1] = lo.y;
    xr[8 * b + 2] = lo.z;
    xr[8 * b + 3] = lo.w;
    xr[8 * b + 4] = hi.x;
    xr[8 * b + 5] = hi.y;
    xr[8 * b + 6] = hi.z;
    xr[8 * b + 7] = hi.w;
  }
  if (round16) {
#pragma unroll
    for (int i = 0; i < 8 * kClNB; ++i) xr[i] = h2f(f2h(xr[i]));
  }
}

// warp_dot32 of one 512-wide fp16 row by the 8 threads of its lane octet:
// thread g accumulates chains j = 0..3 of lane 4g + j (elements 64b + 8g + j,
// then + 4), and the octet forms ((a0+a1)+(a2+a3)) per group, groups summed
// in order.  Every thread of the octet returns the dot.
__device__ __forceinline__ float g8_dot(const uint16_t* w, const float* xr) {
  const int g = threadIdx.x & 7;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int b = 0; b < kClNB; ++b) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + 64 * b + 8 * g);
    float f[8];
    unpack8(wv, f);
    a0 = fmaf(f[0], xr[8 * b], a0);
    a1 = fmaf(f[1], xr[8 * b + 1], a1);
    a2 = fmaf(f[2], xr[8 * b + 2], a2);
    a3 = fmaf(f[3], xr[8 * b + 3], a3);
    a0 = fmaf(f[4], xr[8 * b + 4], a0);
    a1 = fmaf(f[5], xr[8 * b + 5], a1);
    a2 = fmaf(f[6], xr[8 * b + 6], a2);
    a3 = fmaf(f[7], xr[8 * b + 7], a3);
  }
  const float u = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
  const int base = threadIdx.x & 24;
  float s = __shfl_sync(0xffffffffu, u, base);
#pragma unroll
  for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, u, base + j));
  return s;
}

// fp16 activations (values exactly representable in fp16) for the same
// layout, packed: xh[4b + u] = {x[64b + 8g + 2u], x[64b + 8g + 2u + 1]}.
__device__ __forceinline__ void g8h_load_x(const uint16_t* x16, uint32_t* xh) {
  const int g = threadIdx.x & 7;
#pragma unroll
  for (int b = 0; b < kClNB; ++b) {
    const uint4 v = *reinterpret_cast<const uint4*>(x16 + 64 * b + 8 * g);
    xh[4 * b] = v.x;
    xh[4 * b + 1] = v.y;
    xh[4 * b + 2] = v.z;
    xh[4 * b + 3] = v.w;
  }
}
// d = fp32(a) * fp32(b) + c rounded once (the product of two fp16 values is
// exact in fp32), a / b the low or high halves of packed pairs: the same
// result as fmaf(h2f(a), h2f(b), c), without the two conversions.
__device__ __forceinline__ float fma_h_lo(uint32_t a, uint32_t b, float c) {
  float d;
  asm("{\n\t.reg .f16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.f16 %0, a0, b0, %3;\n\t}"
      : "=f"(d)
      : "r"(a), "r"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_h_hi(uint32_t a, uint32_t b, float c) {
  float d;
  asm("{\n\t.reg .f16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.f16 %0, a1, b1, %3;\n\t}"
      : "=f"(d)
      : "r"(a), "r"(b), "f"(c));
  return d;
}
// g8_dot for fp16-exact activations (mixed-precision fma).
__device__ __forceinline__ float g8h_dot(const uint16_t* w, const uint32_t* xh) {
  const int g = threadIdx.x & 7;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int b = 0; b < kClNB; ++b) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + 64 * b + 8 * g);
    a0 = fma_h_lo(wv.x, xh[4 * b], a0);
    a1 = fma_h_hi(wv.x, xh[4 * b], a1);
    a2 = fma_h_lo(wv.y, xh[4 * b + 1], a2);
    a3 = fma_h_hi(wv.y, xh[4 * b + 1], a3);
    a0 = fma_h_lo(wv.z, xh[4 * b + 2], a0);
    a1 = fma_h_hi(wv.z, xh[4 * b + 2], a1);
    a2 = fma_h_lo(wv.w, xh[4 * b + 3], a2);
    a3 = fma_h_hi(wv.w, xh[4 * b + 3], a3);
  }
  const float u = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
  const int base = threadIdx.x & 24;
  float s = __shfl_sync(0xffffffffu, u, base);
#pragma unroll
  for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, u, base + j));
  return s;
}

// Activations of a 2048-wide row in warp_dot32's lane layout:
// xr[2b] = x[64b + o0], xr[2b + 1] = x[64b + o0 + 4].
__device__ __forceinline__ void lane_load_x(const float* x, float* xr) {
  const int lane = threadIdx.x & 31;
  const int o0 = 8 * (lane >> 2) + (lane & 3);
#pragma unroll
  for (int b = 0; b < kClFB; ++b) {
    xr[2 * b] = x[64 * b + o0];
    xr[2 * b + 1] = x[64 * b + o0 + 4];
  }
}
// W2 rows (F = kClF wide) re-ordered once at load so that lane L of a warp
// reads the 64 elements of its warp_dot32 accumulator chain as eight 16-byte
// words, word k at position 32k + L (conflict-free): word k holds, for
// b = 4k .. 4k+3 in order, elements 64b + o0(L) and 64b + o0(L) + 4, with
// o0(L) = 8 (L >> 2) + (L & 3).  One block per row.
__global__ void w2_lane_order_kernel(const uint16_t* __restrict__ w2, uint16_t* __restrict__ out) {
  const size_t row = blockIdx.x;
  const uint16_t* src = w2 + row * kClF;
  uint16_t* dst = out + row * kClF;
  for (int i = threadIdx.x; i < kClF; i += blockDim.x) {
    const int u = i & 7, word = i >> 3;
    const int lane = word & 31, k = word >> 5;
    const int b = 4 * k + (u >> 1);
    const int o0 = 8 * (lane >> 2) + (lane & 3);
    dst[i] = src[64 * b + o0 + 4 * (u & 1)];
  }
}
// warp_dot32 (lane layout, activations in registers: xr[2b] = x[64b + o0],
// xr[2b + 1] = x[64b + o0 + 4]) over a lane-ordered W2 row: the same chain,
// in the same order.
__device__ __forceinline__ float lane_dot_ordered(const uint16_t* w, const float* xr) {
  const int lane = threadIdx.x & 31;
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kClFB / 4; ++k) {
    const uint4 v = w4[32 * k + lane];
    float f[8];
    unpack8(v, f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int b = 4 * k + q;
      acc = fmaf(f[2 * q], xr[2 * b], acc);
      acc = fmaf(f[2 * q + 1], xr[2 * b + 1], acc);
    }
  }
  const float t = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  const float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
  float s = __shfl_sync(0xffffffffu, u, 0);
#pragma unroll
  for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, u, 4 * j));
  return s;
}

// Row slices of this CTA (row_lo over the cluster) and the ring plan.
struct ClSlices {
  int q0, q1, o0, o1, a0, a1, b0, b1, l0, l1;
};
__device__ __forceinline__ ClSlices cl_slices(const T2SDev& m, int cs, int c) {
  ClSlices s;
  s.q0 = row_lo(3 * m.D, cs, c);
  s.q1 = row_lo(3 * m.D, cs, c + 1);
  s.o0 = row_lo(m.D, cs, c);
  s.o1 = row_lo(m.D, cs, c + 1);
  s.a0 = row_lo(m.F, cs, c);
  s.a1 = row_lo(m.F, cs, c + 1);
  s.b0 = row_lo(m.D, cs, c);
  s.b1 = row_lo(m.D, cs, c + 1);
  s.l0 = row_lo(m.V, cs, c);
  s.l1 = row_lo(m.V, cs, c + 1);
  return s;
}
// rows per ring chunk of a matrix with `width` columns
__host__ __device__ constexpr int cl_chunk_rows(int width) {
  return static_cast<int>(kClSlotBytes / (2u * static_cast<uint32_t>(width)));
}

// Copy this CTA's n staged outputs to dst[r0 .. r0+n) in every CTA.
__device__ __forceinline__ void cl_push(const float* stg, float* dst, int r0, int n, int cs) {
  const int tid = threadIdx.x;
  if ((r0 & 3) == 0 && (n & 3) == 0) {
    const int n4 = n >> 2;
    for (int i = tid; i < n4 * cs; i += kClCons) {
      const int d = i / n4, k = i - d * n4;
      *reinterpret_cast<float4*>(cl_map(dst + r0 + 4 * k, static_cast<uint32_t>(d))) =
          reinterpret_cast<const float4*>(stg)[k];
    }
  } else {
    for (int i = tid; i < n * cs; i += kClCons) {
      const int d = i / n, k = i - d * n;
      *cl_map(dst + r0 + k, static_cast<uint32_t>(d)) = stg[k];
    }
  }
}


// The chunk sequence every CTA walks: per step, per layer the chunks of its
// QKV, out, W1 and W2 row slices, then those of its logits slice.
struct ClPlan {
  int nq, no, na, nb, nl;  // chunks per slice
  int per_layer, per_step;
};
__device__ __forceinline__ ClPlan cl_plan(const ClSlices& s, int L, int crD, int crF) {
  ClPlan p;
  p.nq = (s.q1 - s.q0 + crD - 1) / crD;
  p.no = (s.o1 - s.o0 + crD - 1) / crD;
  p.na = (s.a1 - s.a0 + crD - 1) / crD;
  p.nb = (s.b1 - s.b0 + crF - 1) / crF;
  p.nl = (s.l1 - s.l0 + crD - 1) / crD;
  p.per_layer = p.nq + p.no + p.na + p.nb;
  p.per_step = L * p.per_layer + p.nl;
  return p;
}
// Thread 0: bulk-copy chunk c of the sequence into its ring slot.
__device__ void cl_issue(const T2SDev& m, const ClSlices& s, const ClPlan& p, int crD, int crF,
                         uint32_t c, uint8_t* ring, uint64_t* full) {
  const int D = m.D, F = m.F;
  int j = static_cast<int>(c % static_cast<uint32_t>(p.per_step));
  const uint16_t* w;
  int width, r, r1, cr;
  if (j < m.L * p.per_layer) {
    const size_t l = static_cast<size_t>(j / p.per_layer);
    j -= static_cast<int>(l) * p.per_layer;
    if (j < p.nq) {
      w = m.wqkv + l * 3 * D * D; width = D; cr = crD; r = s.q0 + j * crD; r1 = s.q1;
    } else if ((j -= p.nq) < p.no) {
      w = m.wout + l * D * D; width = D; cr = crD; r = s.o0 + j * crD; r1 = s.o1;
    } else if ((j -= p.no) < p.na) {
      w = m.w1 + l * F * D; width = D; cr = crD; r = s.a0 + j * crD; r1 = s.a1;
    } else {
      j -= p.na;
      w = m.w2p + l * D * F; width = F; cr = crF; r = s.b0 + j * crF; r1 = s.b1;
    }
  } else {
    j -= m.L * p.per_layer;
    w = m.wpred; width = D; cr = crD; r = s.l0 + j * crD; r1 = s.l1;
  }
  const uint32_t bytes = static_cast<uint32_t>(min(cr, r1 - r)) * static_cast<uint32_t>(width) * 2u;
  const uint32_t sl = c % kClRing;
  mbar_arrive_expect_tx(&full[sl], bytes);
  bulk_load(ring + static_cast<size_t>(sl) * kClSlotBytes, w + static_cast<size_t>(r) * width, bytes,
            &full[sl]);
}

// Per-thread parameters of "layer set" l (0..L), loaded a phase ahead of
// their use: the bias element tid of layer l's slices (QKV, out, W1, W2 in
// that order), LN1 of layer l and LN2 of layer l - 1 at elements tid and
// tid + kClCons (set L: only the LN2 of the last layer, for the logits).
struct ClParams {
  float bias, g1A, b1A, g1B, b1B, g2A, b2A, g2B, b2B;
};
__device__ __forceinline__ ClParams cl_params(const T2SDev& m, const ClSlices& s, int l, int tid) {
  const int D = m.D, F = m.F;
  ClParams p{};
  const int eA = tid, eB = tid + kClCons;
  if (l < m.L) {
    const int nq = s.q1 - s.q0, no = s.o1 - s.o0, na = s.a1 - s.a0, nb = s.b1 - s.b0;
    const size_t L_ = static_cast<size_t>(l);
    if (tid < nq) p.bias = __ldg(m.bqkv + L_ * 3 * D + s.q0 + tid);
    else if (tid < nq + no) p.bias = __ldg(m.bout + L_ * D + s.o0 + tid - nq);
    else if (tid < nq + no + na) p.bias = __ldg(m.b1 + L_ * F + s.a0 + tid - nq - no);
    else if (tid < nq + no + na + nb) p.bias = __ldg(m.b2 + L_ * D + s.b0 + tid - nq - no - na);
    const float* g = m.n1g + L_ * D;
    const float* b = m.n1b + L_ * D;
    if (eA < D) { p.g1A = __ldg(g + eA); p.b1A = __ldg(b + eA); }
    if (eB < D) { p.g1B = __ldg(g + eB); p.b1B = __ldg(b + eB); }
  }
  if (l > 0) {
    const float* g = m.n2g + static_cast<size_t>(l - 1) * D;
    const float* b = m.n2b + static_cast<size_t>(l - 1) * D;
    if (eA < D) { p.g2A = __ldg(g + eA); p.b2A = __ldg(b + eA); }
    if (eB < D) { p.g2B = __ldg(g + eB); p.b2B = __ldg(b + eB); }
  }
  return p;
}

__global__ void __launch_bounds__(kClThreads, 1)
    t2s_cluster_kernel(const T2SDev m, const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t cl_smem[];
  __shared__ uint64_t full[kClRing];
  __shared__ int done_warps[kClRing];  // warps finished with the slot's current chunk
  __shared__ int tokp[4];

  const int D = m.D, F = m.F, V = m.V, H = m.H, L = m.L;
  constexpr int cs = kClCS;  // the grid is exactly one cluster
  const uint32_t rank = cl_ctarank();
  const ClLayout lay = cl_layout(V);
  uint8_t* ring = cl_smem;
  float* fs = reinterpret_cast<float*>(cl_smem);
  float* xin = fs + lay.xin;
  float* qv = fs + lay.qv;
  float* att = fs + lay.att;
  float* hp = fs + lay.hp;
  float* ffv = fs + lay.ffv;
  float* lg = ffv;  // logits reuse the FFN vector (consumed before they are pushed)
  uint16_t* x16 = reinterpret_cast<uint16_t*>(fs + lay.x16);
  uint16_t* att16 = reinterpret_cast<uint16_t*>(fs + lay.att16);
  uint16_t* hp16 = reinterpret_cast<uint16_t*>(fs + lay.hp16);
  float* bsm = fs + lay.bsm;
  float* stg = fs + lay.stg;
  float* slots = fs + lay.slots;
  float* rec = fs + lay.rec;
  float* red = fs + lay.red;
  uint8_t* seen = reinterpret_cast<uint8_t*>(fs + lay.seen);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ClSlices s = cl_slices(m, cs, static_cast<int>(rank));
  const int crD = cl_chunk_rows(D), crF = cl_chunk_rows(F);
  const ClPlan plan = cl_plan(s, L, crD, crF);
  bool failed = false;
  uint32_t ci = 0;  // chunks consumed

  if (tid == 0) {
    for (int i = 0; i < kClRing; ++i) {
      mbar_init(&full[i], 1);
      done_warps[i] = 0;
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0)
    for (uint32_t c = 0; c < kClRing; ++c) cl_issue(m, s, plan, crD, crF, c, ring, full);
  // chunk ci: wait until it has landed
  auto acquire = [&]() -> const uint16_t* {
    const uint32_t sl = ci % kClRing;
    cl_wait_full(&full[sl], (ci / kClRing) & 1u, m.status, failed);
    return reinterpret_cast<const uint16_t*>(ring + static_cast<size_t>(sl) * kClSlotBytes);
  };
  // this warp is done with chunk ci; the last warp to finish refills the
  // slot with chunk ci + kClRing (no CTA-wide wait per chunk)
  auto release = [&]() {
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();  // the warp's reads of the slot precede its count
      const uint32_t sl = ci % kClRing;
      if (atomicAdd(&done_warps[sl], 1) == kClWarps - 1) {
        done_warps[sl] = 0;
        fence_proxy_async_shared();
        cl_issue(m, s, plan, crD, crF, ci + kClRing, ring, full);
      }
    }
    ++ci;
  };

  const int eos = V - 1;
  for (int c = tid; c < V; c += kClCons) seen[c] = 0;
  cons_sync();
  for (int i = tid; i < a.n_hist; i += kClCons) {
    const int t = a.hist[i];
    if (t >= 0 && t < V) seen[t] = 1;
  }
  for (int i = tid; i < V; i += kClCons) lg[i] = __ldcg(m.logits + i);  // prefill logits
  cons_sync();

  int n_out = 0;
  unsigned long long* tr = nullptr;
#define GSVK_CTR(slot)                                  \
  do {                                                  \
    if (tr && tid == 0) tr[(slot)] = global_ns();       \
  } while (0)
  for (int idx = 0; idx < a.max_steps; ++idx) {
    tr = (a.trace && rank == 0 && idx < kTraceSteps) ? a.trace + idx * kTraceStride : nullptr;
    GSVK_CTR(0);
    ClParams pn = cl_params(m, s, 0, tid);  // layer 0's, in flight during the sampling
    // ------------------------------------------- greedy sample (every CTA)
    const int eos_allowed = idx >= 11;
    const int limit = eos_allowed ? V : V - 1;
    float bv = -INFINITY, sv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = tid; c < limit; c += kClCons) {
      float v = lg[c];
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
    cons_sync();
    if (lane == 0) {
      red[warp] = bv;
      red[kClWarps + warp] = sv;
      reinterpret_cast<int*>(red + 2 * kClWarps)[warp] = bi;
    }
    cons_sync();
    if (tid == 0) {
      float B = red[0], S = red[kClWarps];
      int I = reinterpret_cast<int*>(red + 2 * kClWarps)[0];
      for (int w = 1; w < kClWarps; ++w) {
        const float ov = red[w], os = red[kClWarps + w];
        const int oi = reinterpret_cast<int*>(red + 2 * kClWarps)[w];
        if (ov > B || (ov == B && oi < I)) {
          S = fmaxf(os, B);
          B = ov;
          I = oi;
        } else {
          S = fmaxf(S, ov);
        }
      }
      tokp[0] = I;
      if (rank == 0 && a.margins) a.margins[idx] = __fsub_rn(B, S);
    }
    cons_sync();
    const int tok = tokp[0];
    bool stop = false;
    if (a.stop_on_eos && eos_allowed && tok == eos) {
      stop = true;
    } else {
      if (rank == 0 && tid == 0) a.tokens[n_out] = tok;
      ++n_out;
      if (tid == 0) seen[tok] = 1;
    }
    if (idx + 1 == a.max_steps) stop = true;
    cons_sync();
    GSVK_CTR(1);
    if (stop) break;  // the same step in every CTA

    // ------------------------------------- next input: emb[tok] + alpha*PE
    const int pos = a.pos0 + idx;
    const int len = pos + 1;
    {
      const uint16_t* er = m.emb + static_cast<size_t>(tok) * D;
      const float* pr = m.pe + static_cast<size_t>(a.pe0 + idx) * D;
      for (int i = tid; i < D; i += kClCons) {
        const float v = fmaf(m.alpha, pr[i], h2f(er[i]));
        xin[i] = v;
        x16[i] = f2h(v);
      }
    }
    const int nch = (len + kChunk - 1) / kChunk;
    const int slot = tid >> 6;

    for (int l = 0; l < L; ++l) {
      const uint16_t* kc_l = m.kc + static_cast<size_t>(l) * m.cap * D;
      const uint16_t* vc_l = m.vc + static_cast<size_t>(l) * m.cap * D;
      // --------------------------------------------------------------- P1
      // warm L2 with the K / V rows this thread reads in P2 (all but the new one)
      if (static_cast<int>(rank) < H) {
        const int h = static_cast<int>(rank);
        for (int c = slot; c < nch; c += kClSlots) {
          const int k = c * kChunk + (tid & 63);
          if (k < len - 1) {
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kc_l + static_cast<size_t>(k) * D + h * kClHD));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(vc_l + static_cast<size_t>(k) * D + h * kClHD));
          }
        }
      }
      // this layer's bias slices (loaded a phase ago) and LayerNorm parameters
      const ClParams pc = pn;
      const int nq = s.q1 - s.q0, no = s.o1 - s.o0, na = s.a1 - s.a0, nb = s.b1 - s.b0;
      if (tid < nq + no + na + nb) bsm[tid] = pc.bias;
      cons_sync();
      GSVK_CTR(16 + 16 * l + 0);
      if (l > 0) ln_cons(xin, D, m.eps, red, pc.g2A, pc.b2A, pc.g2B, pc.b2B, x16);  // LN2 of l - 1
      GSVK_CTR(16 + 16 * l + 1);
      {
        uint32_t xh[4 * kClNB];
        g8h_load_x(x16, xh);  // f16(x)
        uint16_t* kl = m.kc + (static_cast<size_t>(l) * m.cap + pos) * D;
        uint16_t* vl = m.vc + (static_cast<size_t>(l) * m.cap + pos) * D;
        for (int r0 = s.q0; r0 < s.q1; r0 += crD) {
          const int nr = min(crD, s.q1 - r0);
          const uint16_t* W = acquire();
          const int rl = 4 * warp + (lane >> 3);
          if (4 * warp < nr) {
            const int rr = rl < nr ? rl : 0;
            const float acc = g8h_dot(W + static_cast<size_t>(rr) * D, xh);
            if (rl < nr && (lane & 7) == 0) {
              const int r = r0 + rl;
              const float v = __fadd_rn(acc, bsm[r - s.q0]);
              if (r < D)
                stg[r - s.q0] = v;
              else if (r < 2 * D)
                kl[r - D] = f2h(v);
              else
                vl[r - 2 * D] = f2h(v);
            }
          }
          release();
        }
      }
      cons_sync();
      GSVK_CTR(16 + 16 * l + 2);
      if (s.q0 < D) cl_push(stg, qv, s.q0, min(s.q1, D) - s.q0, cs);
      cl_barrier_all();
      GSVK_CTR(16 + 16 * l + 3);
      // --------------------------------------------------------------- P2
      pn = cl_params(m, s, l + 1, tid);  // the next layer's (or the logits') parameters
      // CTA h: head h's key chunks over its attention slots, records kept
      // locally, then the head's merge (canonical chunk order)
      if (static_cast<int>(rank) < H) {
        const int h = static_cast<int>(rank);
        float* sm = slots + slot * slot_floats<kClHD>();
        for (int c = slot; c < nch; c += kClSlots) {
          const int k0 = c * kChunk, k1 = min(len, k0 + kChunk);
          attn_chunk_slot<kClHD>(qv + h * kClHD, false, kc_l + h * kClHD, vc_l + h * kClHD, D, k0,
                                 k1, m.scale, sm, 2 + slot, rec + c * rec_floats<kClHD>());
        }
      }
      cons_sync();
      GSVK_CTR(16 + 16 * l + 4);
      GSVK_CTR(16 + 16 * l + 5);
      if (static_cast<int>(rank) < H && warp == 0) {
        float o0, o1;
        attn_combine<kClHD>(rec, nch, false, &o0, &o1);
        const uint16_t v16 = f2h(o0);
        const float v = h2f(v16);
        for (int d = 0; d < cs; ++d) {
          *cl_map(att + rank * kClHD + lane, static_cast<uint32_t>(d)) = v;
          *cl_map(att16 + rank * kClHD + lane, static_cast<uint32_t>(d)) = v16;
        }
      }
      cl_barrier_all();
      GSVK_CTR(16 + 16 * l + 6);
      // --------------------------------------------------------------- P3
      {
        uint32_t xh[4 * kClNB];
        g8h_load_x(att16, xh);  // head outputs, fp16 values
        for (int r0 = s.o0; r0 < s.o1; r0 += crD) {
          const int nr = min(crD, s.o1 - r0);
          const uint16_t* W = acquire();
          const int rl = 4 * warp + (lane >> 3);
          if (4 * warp < nr) {
            const int rr = rl < nr ? rl : 0;
            const float acc = g8h_dot(W + static_cast<size_t>(rr) * D, xh);
            if (rl < nr && (lane & 7) == 0) {
              const int r = r0 + rl;
              stg[r - s.o0] = __fadd_rn(__fadd_rn(acc, bsm[nq + r - s.o0]), xin[r]);
            }
          }
          release();
        }
      }
      cons_sync();
      cl_push(stg, hp, s.o0, s.o1 - s.o0, cs);
      GSVK_CTR(16 + 16 * l + 7);
      cl_barrier_all();
      GSVK_CTR(16 + 16 * l + 8);
      // --------------------------------------------------------------- P4
      ln_cons(hp, D, m.eps, red, pc.g1A, pc.b1A, pc.g1B, pc.b1B, hp16);  // h = LN1(hpre)
      GSVK_CTR(16 + 16 * l + 9);
      {
        uint32_t xh[4 * kClNB];
        g8h_load_x(hp16, xh);  // f16(h)
        for (int r0 = s.a0; r0 < s.a1; r0 += crD) {
          const int nr = min(crD, s.a1 - r0);
          const uint16_t* W = acquire();
          const int rl = 4 * warp + (lane >> 3);
          if (4 * warp < nr) {
            const int rr = rl < nr ? rl : 0;
            const float acc = g8h_dot(W + static_cast<size_t>(rr) * D, xh);
            if (rl < nr && (lane & 7) == 0) {
              const int r = r0 + rl;
              const float v = __fadd_rn(acc, bsm[nq + no + r - s.a0]);
              stg[r - s.a0] = v > 0.f ? v : 0.f;
            }
          }
          release();
        }
      }
      cons_sync();
      cl_push(stg, ffv, s.a0, s.a1 - s.a0, cs);
      GSVK_CTR(16 + 16 * l + 10);
      cl_barrier_all();
      GSVK_CTR(16 + 16 * l + 11);
      // --------------------------------------------------------------- P5
      {
        float xr[2 * kClFB];
        lane_load_x(ffv, xr);
        for (int r0 = s.b0; r0 < s.b1; r0 += crF) {
          const int nr = min(crF, s.b1 - r0);
          const uint16_t* W = acquire();
          if (warp < nr) {
            const float acc = lane_dot_ordered(W + static_cast<size_t>(warp) * F, xr);
            if (lane == 0) {
              const int r = r0 + warp;
              stg[r - s.b0] = __fadd_rn(__fadd_rn(acc, bsm[nq + no + na + r - s.b0]), hp[r]);
            }
          }
          release();
        }
      }
      cons_sync();
      cl_push(stg, xin, s.b0, s.b1 - s.b0, cs);
      GSVK_CTR(16 + 16 * l + 12);
      cl_barrier_all();
      GSVK_CTR(16 + 16 * l + 13);
    }
    // ------------------------------------------------------------- logits
    ln_cons(xin, D, m.eps, red, pn.g2A, pn.b2A, pn.g2B, pn.b2B, nullptr);  // final LN2
    {
      float xr[8 * kClNB];
      g8_load_x(xin, xr, false);
      for (int r0 = s.l0; r0 < s.l1; r0 += crD) {
        const int nr = min(crD, s.l1 - r0);
        const uint16_t* W = acquire();
        const int rl = 4 * warp + (lane >> 3);
        if (4 * warp < nr) {
          const int rr = rl < nr ? rl : 0;
          const float acc = g8_dot(W + static_cast<size_t>(rr) * D, xr);
          if (rl < nr && (lane & 7) == 0) {
            stg[r0 + rl - s.l0] = acc;
            m.logits[r0 + rl] = acc;  // the last step's logits stay readable on the host
          }
        }
        release();
      }
    }
    cons_sync();
    cl_push(stg, lg, s.l0, s.l1 - s.l0, cs);
    GSVK_CTR(2);
    cl_barrier_all();
    GSVK_CTR(3);
  }
#undef GSVK_CTR
  // the chunks issued beyond the last one consumed must land before exit
  // (one thread, bounded; no warp-collective operation here)
  cons_sync();
  if (tid == 0) {
    for (uint32_t k = ci; k < ci + kClRing && !failed; ++k) {
      bool ok = false;
      for (uint32_t i = 0; i < kSpinLimit && !ok; ++i)
        ok = mbar_test(&full[k % kClRing], (k / kClRing) & 1u);
      if (!ok) {
        atomicExch(m.status, DEV_TIMEOUT);
        failed = true;
      }
    }
    if (rank == 0 && a.n_out) *a.n_out = n_out;
  }
  __syncthreads();
  cl_barrier_all();  // no CTA leaves while another may still write its shared memory
}
