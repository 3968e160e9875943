// oracle.cpp — CPU restatement of the reference `src/kern` hot path and its
// callers.  TEST INFRASTRUCTURE: the parity checker and the timed CPU
// baseline; the CUDA product path never links it.
//
// Built with -ffp-contract=off so that every fused multiply-add below is an
// explicit fmaf() exactly where the reference issues one (vfmaq_f32 /
// vfmlalq_*), and every separate multiply/add is rounded separately where the
// reference rounds separately (vmulq_f32 + vaddq_f32).
//
// NEON horizontal sums (vaddvq_f32) are restated as (l0 + l1) + (l2 + l3),
// the AArch64 FADDP pairwise order.
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <mutex>
#include <thread>
#include <random>
#include <vector>

namespace {

// ---------------------------------------------------------------- fp16 bits
inline float h2f(uint16_t b) {
  _Float16 h;
  std::memcpy(&h, &b, 2);
  return static_cast<float>(h);
}
inline uint16_t f2h(float v) {
  const _Float16 h = static_cast<_Float16>(v);  // IEEE RNE
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}
inline float round_f16(float v) { return h2f(f2h(v)); }

inline float vaddv4(const float* l) { return (l[0] + l[1]) + (l[2] + l[3]); }

// ---------------------------------------------------------------- thread pool
// Persistent workers pulling fixed-size chunks; the restatement of
// rt::parallel_for (runtime/threadpool.hpp:141).  Results never depend on the
// partition: every output element is computed by exactly one chunk with a
// fixed arithmetic order.
class Pool {
 public:
  ~Pool() { resize(0); }

  void resize(int n) {
    {
      std::unique_lock<std::mutex> lk(mu_);
      quit_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
    th_.clear();
    quit_ = false;
    nthreads_ = std::max(1, n);
    for (int i = 1; i < nthreads_; ++i) th_.emplace_back([this] { loop(); });
  }
  int size() const { return nthreads_; }

  void run(size_t n, size_t grain, const std::function<void(size_t, size_t)>& fn) {
    if (n == 0) return;
    if (grain == 0) grain = 1;
    if (nthreads_ <= 1 || n <= grain) {
      fn(0, n);
      return;
    }
    std::unique_lock<std::mutex> call_lk(call_mu_);
    {
      std::unique_lock<std::mutex> lk(mu_);
      fn_ = &fn;
      n_ = n;
      grain_ = grain;
      next_.store(0);
      active_ = static_cast<int>(th_.size());
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return active_ == 0; });
    fn_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      const size_t b = next_.fetch_add(grain_);
      if (b >= n_) break;
      (*fn_)(b, std::min(n_, b + grain_));
    }
  }
  void loop() {
    uint64_t seen = 0;
    {
      std::unique_lock<std::mutex> lk(mu_);
      seen = gen_;
    }
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (quit_) return;
      }
      work();
      std::unique_lock<std::mutex> lk(mu_);
      if (--active_ == 0) done_cv_.notify_all();
    }
  }

  std::vector<std::thread> th_;
  std::mutex mu_, call_mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t, size_t)>* fn_ = nullptr;
  size_t n_ = 0, grain_ = 1;
  std::atomic<size_t> next_{0};
  int active_ = 0;
  uint64_t gen_ = 0;
  bool quit_ = false;
  int nthreads_ = 1;
};

Pool& pool() {
  static Pool p;
  return p;
}

// Row-band split over all workers: grain = ceil(rows / workers)
// (gemv.cpp:117-126, gemv_fmlal.cpp:117-129).
void row_bands(size_t rows, const std::function<void(size_t, size_t)>& fn) {
  const size_t workers = static_cast<size_t>(pool().size());
  const size_t grain = (rows + workers - 1) / workers;
  pool().run(rows, grain, fn);
}

// ------------------------------------------------ gemv_f16w_f32acc (gemv.cpp)
// gemv.cpp:36-109: 4 rows at a time, each row with two 4-lane accumulators
// fed by FMA over 8-element chunks, scalar FMA tail.
void gemv_f16w_rows(const uint16_t* w, const float* x, float* y, size_t rb,
                    size_t re, size_t in) {
  const size_t vec_end = in & ~size_t{7};
  size_t r = rb;
  for (; r + 4 <= re; r += 4) {
    float acc[4][8];
    for (auto& a : acc)
      for (float& v : a) v = 0.f;
    for (size_t i = 0; i < vec_end; i += 8) {
      for (int q = 0; q < 4; ++q) {
        const uint16_t* wr = w + (r + q) * in + i;
        for (int l = 0; l < 8; ++l) acc[q][l] = std::fmaf(h2f(wr[l]), x[i + l], acc[q][l]);
      }
    }
    float s[4];
    for (int q = 0; q < 4; ++q) {
      float t[4];
      for (int l = 0; l < 4; ++l) t[l] = acc[q][l] + acc[q][4 + l];  // vaddq
      s[q] = vaddv4(t);
    }
    for (size_t i = vec_end; i < in; ++i)
      for (int q = 0; q < 4; ++q) s[q] = std::fmaf(h2f(w[(r + q) * in + i]), x[i], s[q]);
    for (int q = 0; q < 4; ++q) y[r + q] = s[q];
  }
  for (; r < re; ++r) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const uint16_t* wr = w + r * in;
    for (size_t i = 0; i < vec_end; i += 8)
      for (int l = 0; l < 8; ++l) a[l] = std::fmaf(h2f(wr[i + l]), x[i + l], a[l]);
    float s = vaddv4(a) + vaddv4(a + 4);
    for (size_t i = vec_end; i < in; ++i) s = std::fmaf(h2f(wr[i]), x[i], s);
    y[r] = s;
  }
}

// ------------------------------------------- gemv_f16x_fmlal (gemv_fmlal.cpp)
// gemv_fmlal.cpp:40-109: 8 accumulators x 4 lanes over 64-element steps; each
// accumulator takes the low then the high half of its 8-element slice.
float row_dot_fmlal(const uint16_t* wr, const uint16_t* xh, size_t in) {
  const size_t vec_end = in & ~size_t{63};
  float a[8][4];
  for (auto& v : a)
    for (float& z : v) z = 0.f;
  size_t i = 0;
  for (; i < vec_end; i += 64) {
    for (int j = 0; j < 8; ++j) {
      const size_t o = i + 8 * j;
      for (int l = 0; l < 4; ++l) a[j][l] = std::fmaf(h2f(wr[o + l]), h2f(xh[o + l]), a[j][l]);
      for (int l = 0; l < 4; ++l)
        a[j][l] = std::fmaf(h2f(wr[o + 4 + l]), h2f(xh[o + 4 + l]), a[j][l]);
    }
  }
  float s = vaddv4(a[0]);
  for (int j = 1; j < 8; ++j) s = s + vaddv4(a[j]);
  for (; i < in; ++i) s = std::fmaf(h2f(wr[i]), h2f(xh[i]), s);  // exact product, one rounding
  return s;
}

// The same association with fp32 activations: the canonical order of every
// T2S dot product (GEMV and prefill GEMM alike), so that the device kernels can
// reproduce each sum bit for bit (32 accumulators = 32 lanes of a warp).
float dot32(const uint16_t* wr, const float* x, size_t in) {
  const size_t vec_end = in & ~size_t{63};
  float a[8][4];
  for (auto& v : a)
    for (float& z : v) z = 0.f;
  size_t i = 0;
  for (; i < vec_end; i += 64)
    for (int j = 0; j < 8; ++j) {
      const size_t o = i + 8 * j;
      for (int l = 0; l < 4; ++l) a[j][l] = std::fmaf(h2f(wr[o + l]), x[o + l], a[j][l]);
      for (int l = 0; l < 4; ++l) a[j][l] = std::fmaf(h2f(wr[o + 4 + l]), x[o + 4 + l], a[j][l]);
    }
  float s = vaddv4(a[0]);
  for (int j = 1; j < 8; ++j) s = s + vaddv4(a[j]);
  for (; i < in; ++i) s = std::fmaf(h2f(wr[i]), x[i], s);
  return s;
}

// y[r] = dot32(W[r], x) over row bands.
void gemv32(const uint16_t* w, const float* x, float* y, size_t out, size_t in) {
  row_bands(out, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; ++r) y[r] = dot32(w + r * in, x, in);
  });
}

// Deterministic exp for the softmax: Cody-Waite reduction x = n ln2 + r with
// the two-constant split of ln 2, then the degree-7 Taylor polynomial of e^r
// (|r| <= ln2/2, truncation < 6e-9 relative) in Horner form, scaled by 2^n
// through the exponent field.  Written with explicit fmaf so the CUDA build
// produces the same bits; within 2 ulp of libm expf.
float exp_det(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) return INFINITY;
  const float n = std::rint(x * 1.44269504088896341f);
  float r = std::fmaf(n, -0.693359375f, x);
  r = std::fmaf(n, 2.12194440e-4f, r);
  float p = 1.98412698e-4f;
  p = std::fmaf(p, r, 1.38888889e-3f);
  p = std::fmaf(p, r, 8.33333333e-3f);
  p = std::fmaf(p, r, 4.16666667e-2f);
  p = std::fmaf(p, r, 1.66666667e-1f);
  p = std::fmaf(p, r, 0.5f);
  p = std::fmaf(p, r, 1.0f);
  p = std::fmaf(p, r, 1.0f);
  const int ni = static_cast<int>(n);
  uint32_t bits = static_cast<uint32_t>(ni + 127) << 23;
  float scale;
  std::memcpy(&scale, &bits, 4);
  return p * scale;
}

// -------------------------------------------- gemm_f16x_fmlal tile4 kernel
// gemv_fmlal.cpp:140-185: per (m, n) one 4-lane accumulator; 8-element K
// steps (low then high half), the K tail accumulated into lane 0.
void gemm_f16_tile4(const uint16_t* a, const uint16_t* b, float* c, size_t M,
                    size_t N, size_t K) {
  const size_t vec_end = K & ~size_t{7};
  for (size_t m = 0; m < M; ++m) {
    const uint16_t* ar = a + m * K;
    for (size_t n = 0; n < N; ++n) {
      const uint16_t* br = b + n * K;
      float acc[4] = {0, 0, 0, 0};
      for (size_t k = 0; k < vec_end; k += 8) {
        for (int l = 0; l < 4; ++l) acc[l] = std::fmaf(h2f(ar[k + l]), h2f(br[k + l]), acc[l]);
        for (int l = 0; l < 4; ++l)
          acc[l] = std::fmaf(h2f(ar[k + 4 + l]), h2f(br[k + 4 + l]), acc[l]);
      }
      for (size_t k = vec_end; k < K; ++k) acc[0] = acc[0] + h2f(ar[k]) * h2f(br[k]);
      c[m * N + n] = vaddv4(acc);
    }
  }
}

// fp32 dot with one FMA chain (the restated sgemm kernel).
inline float dot_f32_f16w(const uint16_t* w, const float* x, size_t n) {
  float s = 0.f;
  for (size_t i = 0; i < n; ++i) s = std::fmaf(h2f(w[i]), x[i], s);
  return s;
}

// --------------------------------------------------------- T2S attention dots
// t2s_engine.cpp:69-99 dot_f16kv: 4 accumulators x 4 lanes over 16-element
// chunks, tree (a0+a1)+(a2+a3), then (s0+s2)+(s1+s3).
float dot_f16kv(const float* q, const uint16_t* k16, size_t HD) {
  float a[4][4];
  for (auto& v : a)
    for (float& z : v) z = 0.f;
  size_t e = 0;
  for (; e + 16 <= HD; e += 16)
    for (int j = 0; j < 4; ++j)
      for (int l = 0; l < 4; ++l)
        a[j][l] = std::fmaf(q[e + 4 * j + l], h2f(k16[e + 4 * j + l]), a[j][l]);
  float s[4];
  for (int l = 0; l < 4; ++l) s[l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
  float dot = (s[0] + s[2]) + (s[1] + s[3]);
  for (; e < HD; ++e) dot = std::fmaf(q[e], h2f(k16[e]), dot);
  return dot;
}

// t2s_engine.cpp:126-145 accum_f16kv: ov += p * v with separate mul and add.
void accum_f16kv(float* ov, const uint16_t* v16, float p, size_t HD) {
  for (size_t e = 0; e < HD; ++e) {
    const float t = p * h2f(v16[e]);
    ov[e] = ov[e] + t;
  }
}

constexpr size_t kAttnChunk = 64;

// Attention of one query row q (fp32, one head) over key/value slots
// [0, n) of a token-major fp16 cache (t2s_engine.cpp:1062-1087): scores
// dot_f16kv * scale, stable softmax, probability-weighted sum of V.  The
// softmax is associated in fixed chunks of 64 slots from slot 0 (per chunk
// max m_c, sum l_c of exp(s - m_c) and o_c = sum exp(s - m_c) v, each a
// sequential sum in slot order; then chunk weights exp(m_c - M)), the order a
// split-K device kernel reproduces exactly; it equals the reference's softmax
// up to reassociation.  out receives HD values.
void attend_canon(const float* q, const uint16_t* kc, const uint16_t* vc, size_t D, size_t n,
                  size_t HD, float scale, float* out) {
  const size_t nch = (n + kAttnChunk - 1) / kAttnChunk;
  std::vector<float> mc(nch), lc(nch), oc(nch * HD, 0.f), sc(kAttnChunk);
  for (size_t c = 0; c < nch; ++c) {
    const size_t k0 = c * kAttnChunk, k1 = std::min(n, k0 + kAttnChunk);
    float m = -INFINITY;
    for (size_t k = k0; k < k1; ++k) {
      sc[k - k0] = dot_f16kv(q, kc + k * D, HD) * scale;
      m = m < sc[k - k0] ? sc[k - k0] : m;
    }
    float l = 0.f;
    float* o = oc.data() + c * HD;
    for (size_t k = k0; k < k1; ++k) {
      const float e = exp_det(sc[k - k0] - m);
      l = l + e;
      accum_f16kv(o, vc + k * D, e, HD);
    }
    mc[c] = m;
    lc[c] = l;
  }
  float M = -INFINITY;
  for (size_t c = 0; c < nch; ++c) M = M < mc[c] ? mc[c] : M;
  float L = 0.f;
  for (size_t e = 0; e < HD; ++e) out[e] = 0.f;
  for (size_t c = 0; c < nch; ++c) {
    const float w = exp_det(mc[c] - M);
    L = L + lc[c] * w;
    for (size_t e = 0; e < HD; ++e) out[e] = out[e] + oc[c * HD + e] * w;
  }
  const float inv = 1.0f / L;
  for (size_t e = 0; e < HD; ++e) out[e] = out[e] * inv;
}

// y[T,out] = act(dot32(W[o], f16(x[t])) + b) (prefill projections).
void linear_canon(const float* x, size_t T, size_t in, const uint16_t* w, size_t out,
                  const float* bias, bool relu, float* y) {
  std::vector<float> xr(T * in);
  for (size_t i = 0; i < T * in; ++i) xr[i] = round_f16(x[i]);
  pool().run(T * out, 64, [&](size_t b, size_t e) {
    for (size_t idx = b; idx < e; ++idx) {
      const size_t t = idx / out, o = idx % out;
      float v = dot32(w + o * in, xr.data() + t * in, in);
      if (bias) v = v + bias[o];
      if (relu) v = v > 0.f ? v : 0.f;
      y[idx] = v;
    }
  });
}

}  // namespace

extern "C" {

void ora_set_threads(int n) { pool().resize(n); }
int ora_get_threads(void) { return pool().size(); }

void ora_f32_to_f16(const float* src, uint16_t* dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = f2h(src[i]);
}
void ora_f16_to_f32(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = h2f(src[i]);
}

void ora_gemv_f16w_f32acc_ref(const uint16_t* w, const float* x, float* y, size_t out,
                              size_t in) {
  for (size_t r = 0; r < out; ++r) {
    float s = 0.f;
    for (size_t i = 0; i < in; ++i) s = s + h2f(w[r * in + i]) * x[i];
    y[r] = s;
  }
}

void ora_gemv_f16w_f32acc(const uint16_t* w, const float* x, float* y, size_t out, size_t in) {
  if (out * in < (size_t{1} << 18)) {  // gemv.cpp:114
    gemv_f16w_rows(w, x, y, 0, out, in);
    return;
  }
  row_bands(out, [&](size_t b, size_t e) { gemv_f16w_rows(w, x, y, b, e, in); });
}

void ora_gemv_f16x_fmlal(const uint16_t* w, const uint16_t* xh, float* y, size_t out,
                         size_t in) {
  if (out * in < (size_t{1} << 18)) {  // gemv_fmlal.cpp:116
    for (size_t r = 0; r < out; ++r) y[r] = row_dot_fmlal(w + r * in, xh, in);
    return;
  }
  row_bands(out, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; ++r) y[r] = row_dot_fmlal(w + r * in, xh, in);
  });
}

void ora_gemm_f16x_fmlal(const uint16_t* a, const uint16_t* b, float* c, size_t M, size_t N,
                         size_t K) {
  if (M * N * K < (size_t{1} << 20)) {  // gemv_fmlal.cpp:190
    gemm_f16_tile4(a, b, c, M, N, K);
    return;
  }
  const size_t workers = static_cast<size_t>(pool().size());
  size_t mblock = (M + workers - 1) / workers;
  mblock = (mblock + 3) & ~size_t{3};  // gemv_fmlal.cpp:197
  pool().run(M, mblock, [&](size_t mb, size_t me) {
    gemm_f16_tile4(a + mb * K, b, c + mb * N, me - mb, N, K);
  });
}

void ora_sgemm(char transa, char transb, int M, int N, int K, float alpha, const float* A,
               int lda, const float* B, int ldb, float beta, float* C, int ldc) {
  const bool ta = transa == 'T' || transa == 't';
  const bool tb = transb == 'T' || transb == 't';
  pool().run(static_cast<size_t>(M), 1, [&](size_t mb, size_t me) {
    for (size_t i = mb; i < me; ++i)
      for (int j = 0; j < N; ++j) {
        float s = 0.f;
        for (int k = 0; k < K; ++k) {
          const float av = ta ? A[static_cast<size_t>(k) * lda + i] : A[i * lda + k];
          const float bv = tb ? B[static_cast<size_t>(j) * ldb + k] : B[static_cast<size_t>(k) * ldb + j];
          s = std::fmaf(av, bv, s);
        }
        float& cv = C[i * ldc + j];
        cv = beta == 0.f ? alpha * s : alpha * s + beta * cv;
      }
  });
}

// ----------------------------------------------------------------- primitives
void ora_layernorm(const float* x, const float* g, const float* b, float* y, size_t n,
                   double eps) {
  const size_t vec_end = n & ~size_t{7};
  float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0}, q0[4] = {0, 0, 0, 0}, q1[4] = {0, 0, 0, 0};
  size_t i = 0;
  for (; i < vec_end; i += 8)
    for (int l = 0; l < 4; ++l) {
      s0[l] = s0[l] + x[i + l];
      s1[l] = s1[l] + x[i + 4 + l];
      q0[l] = std::fmaf(x[i + l], x[i + l], q0[l]);
      q1[l] = std::fmaf(x[i + 4 + l], x[i + 4 + l], q1[l]);
    }
  double sum = static_cast<double>(vaddv4(s0) + vaddv4(s1));
  double sqsum = static_cast<double>(vaddv4(q0) + vaddv4(q1));
  for (; i < n; ++i) {
    sum += x[i];
    sqsum += static_cast<double>(x[i]) * x[i];
  }
  const double dn = static_cast<double>(n);
  const float mean = static_cast<float>(sum / dn);
  float var = static_cast<float>(sqsum / dn - static_cast<double>(mean) * mean);
  if (!(var >= 0.0f)) {  // kern.cpp:45-52 two-pass fallback
    double s2 = 0;
    for (size_t j = 0; j < n; ++j) {
      const double d = static_cast<double>(x[j]) - mean;
      s2 += d * d;
    }
    var = static_cast<float>(s2 / dn);
  }
  const float rstd = static_cast<float>(1.0 / std::sqrt(static_cast<double>(var) + eps));
  for (size_t j = 0; j < n; ++j) y[j] = std::fmaf((x[j] - mean) * rstd, g[j], b[j]);
}

void ora_rmsnorm(const float* x, const float* g, float* y, size_t n, double eps) {
  const size_t vec_end = n & ~size_t{7};
  float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
  size_t i = 0;
  for (; i < vec_end; i += 8)
    for (int l = 0; l < 4; ++l) {
      s0[l] = std::fmaf(x[i + l], x[i + l], s0[l]);
      s1[l] = std::fmaf(x[i + 4 + l], x[i + 4 + l], s1[l]);
    }
  float ss = vaddv4(s0) + vaddv4(s1);
  for (; i < n; ++i) ss = ss + x[i] * x[i];
  const float inv_rms = static_cast<float>(1.0 / std::sqrt(ss / static_cast<double>(n) + eps));
  for (size_t j = 0; j < n; ++j) y[j] = x[j] * inv_rms * g[j];
}

void ora_softmax(const float* x, float* y, size_t n) {
  float m = x[0];
  for (size_t i = 1; i < n; ++i) m = m < x[i] ? x[i] : m;
  float sum = 0.f;
  for (size_t i = 0; i < n; ++i) {
    const float e = std::exp(x[i] - m);
    y[i] = e;
    sum = sum + e;
  }
  const float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) y[i] = y[i] * inv;
}

void ora_relu(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}
void ora_silu(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = x[i] / (1.0f + std::exp(-x[i]));
}
void ora_gelu_erf(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = 0.5f * x[i] * (1.f + std::erf(x[i] * 0.70710678118654752440f));
}
void ora_leaky_relu(const float* x, float* y, size_t n, float slope) {
  for (size_t i = 0; i < n; ++i) y[i] = x[i] < 0.f ? x[i] * slope : x[i];
}

static void apply_act(float* v, size_t n, int act, float slope) {
  switch (act) {
    case ORA_ACT_RELU: ora_relu(v, v, n); break;
    case ORA_ACT_GELU_ERF: ora_gelu_erf(v, v, n); break;
    case ORA_ACT_LEAKY: ora_leaky_relu(v, v, n, slope); break;
    default: break;
  }
}

void ora_linear_f16(const float* x, size_t T, size_t in, const uint16_t* w, size_t out,
                    const float* bias, int act, float slope, float* y) {
  std::vector<uint16_t> xh(T * in);
  ora_f32_to_f16(x, xh.data(), T * in);
  ora_gemm_f16x_fmlal(xh.data(), w, y, T, out, in);
  if (bias)
    for (size_t t = 0; t < T; ++t)
      for (size_t o = 0; o < out; ++o) y[t * out + o] = y[t * out + o] + bias[o];
  apply_act(y, T * out, act, slope);
}

// ---------------------------------------------------------------- convolutions
void ora_conv1d(const float* x, size_t Ci, size_t T, const uint16_t* w, const float* bias,
                size_t Co, size_t k, size_t dil, int round_in, float* y) {
  const size_t K = Ci * k;
  const long long pad_l = static_cast<long long>((k - 1) * dil) / 2;  // conv1d.hpp:165
  // im2col col[(i*k+kk), t] (conv1d.hpp:166-176), optionally fp16-rounded.
  std::vector<float> col(K * T);
  for (size_t i = 0; i < Ci; ++i)
    for (size_t kk = 0; kk < k; ++kk)
      for (size_t t = 0; t < T; ++t) {
        const long long src = static_cast<long long>(t) + static_cast<long long>(kk * dil) - pad_l;
        float v = (src >= 0 && src < static_cast<long long>(T)) ? x[i * T + src] : 0.f;
        col[(i * k + kk) * T + t] = round_in ? round_f16(v) : v;
      }
  std::vector<float> wf(Co * K);
  ora_f16_to_f32(w, wf.data(), Co * K);
  pool().run(Co, 1, [&](size_t cb, size_t ce) {
    std::vector<float> acc(T);
    for (size_t o = cb; o < ce; ++o) {
      std::fill(acc.begin(), acc.end(), 0.f);
      for (size_t kk = 0; kk < K; ++kk) {
        const float wv = wf[o * K + kk];
        const float* cr = col.data() + kk * T;
        for (size_t t = 0; t < T; ++t) acc[t] = std::fmaf(wv, cr[t], acc[t]);
      }
      const float bv = bias ? bias[o] : 0.f;
      for (size_t t = 0; t < T; ++t) y[o * T + t] = acc[t] + bv;  // add_bias (conv1d.hpp:196)
    }
  });
}

void ora_convt1d(const float* x, size_t Ci, size_t T, const uint16_t* w, const float* bias,
                 size_t Co, size_t k, size_t u, int round_in, float* y) {
  const long long pad = static_cast<long long>((k - u) / 2);  // conv1d.hpp:263
  const size_t Tout = T * u;
  std::vector<float> xr(Ci * T);
  for (size_t i = 0; i < Ci * T; ++i) xr[i] = round_in ? round_f16(x[i]) : x[i];
  // phase weights wd[d][o][i] = W[i,o,d] (conv1d.hpp:226-232)
  std::vector<float> wd(k * Co * Ci);
  for (size_t d = 0; d < k; ++d)
    for (size_t o = 0; o < Co; ++o)
      for (size_t i = 0; i < Ci; ++i) wd[(d * Co + o) * Ci + i] = h2f(w[(i * Co + o) * k + d]);
  pool().run(Co, 1, [&](size_t cb, size_t ce) {
    std::vector<float> tmp(T);
    for (size_t o = cb; o < ce; ++o) {
      float* yr = y + o * Tout;
      std::fill(yr, yr + Tout, 0.f);  // y.reset (conv1d.hpp:265)
      for (size_t d = 0; d < k; ++d) {
        // phase GEMM row: tmp[j] = sum_i wd[d][o][i] * x[i][j]
        std::fill(tmp.begin(), tmp.end(), 0.f);
        for (size_t i = 0; i < Ci; ++i) {
          const float wv = wd[(d * Co + o) * Ci + i];
          const float* xi = xr.data() + i * T;
          for (size_t j = 0; j < T; ++j) tmp[j] = std::fmaf(wv, xi[j], tmp[j]);
        }
        // scatter_raw (conv1d.hpp:347-359)
        for (size_t j = 0; j < T; ++j) {
          const long long opos = static_cast<long long>(j * u + d) - pad;
          if (opos < 0 || opos >= static_cast<long long>(Tout)) continue;
          yr[opos] = yr[opos] + tmp[j];
        }
      }
      const float bv = bias ? bias[o] : 0.f;
      for (size_t t = 0; t < Tout; ++t) yr[t] = yr[t] + bv;
    }
  });
}

size_t ora_decoder_out_len(const ora_decoder_cfg* cfg, size_t T) {
  size_t t = T;
  for (int s = 0; s < cfg->n_stages; ++s) t *= static_cast<size_t>(cfg->up_rate[s]);
  return t;
}

void ora_decoder_forward(const ora_decoder_cfg* cfg, const uint16_t* const* w,
                         const float* const* b, const float* z, size_t T, int round_in,
                         float* wav) {
  size_t C = static_cast<size_t>(cfg->ch0);
  size_t L = T;
  std::vector<float> x(C * L);
  ora_conv1d(z, cfg->in_ch, T, w[0], b[0], C, cfg->conv_pre_k, 1, round_in, x.data());
  const float kInv = 1.f / 3.f;
  for (int s = 0; s < cfg->n_stages; ++s) {
    const size_t base = 1 + static_cast<size_t>(s) * 19;
    ora_leaky_relu(x.data(), x.data(), x.size(), cfg->lrelu_slope);
    const size_t Cn = C / 2, Ln = L * cfg->up_rate[s];
    std::vector<float> xu(Cn * Ln);
    ora_convt1d(x.data(), C, L, w[base], b[base], Cn, cfg->up_k[s], cfg->up_rate[s], round_in,
                xu.data());
    C = Cn;
    L = Ln;
    std::vector<float> sum(C * L), cur(C * L), tin(C * L), ta(C * L), tb(C * L);
    for (int j = 0; j < 3; ++j) {  // dec.hpp:303-335 serial resblock path
      cur = xu;
      for (int p = 0; p < 3; ++p) {
        const size_t i1 = base + 1 + j * 6 + p * 2;
        ora_leaky_relu(cur.data(), tin.data(), cur.size(), cfg->lrelu_slope);
        ora_conv1d(tin.data(), C, L, w[i1], b[i1], C, cfg->res_k[j], cfg->res_dil[p], round_in,
                   ta.data());
        ora_leaky_relu(ta.data(), ta.data(), ta.size(), cfg->lrelu_slope);
        ora_conv1d(ta.data(), C, L, w[i1 + 1], b[i1 + 1], C, cfg->res_k[j], 1, round_in,
                   tb.data());
        for (size_t i = 0; i < cur.size(); ++i) cur[i] = cur[i] + tb[i];
      }
      if (j == 0)
        for (size_t i = 0; i < sum.size(); ++i) sum[i] = cur[i] * kInv;
      else
        for (size_t i = 0; i < sum.size(); ++i) sum[i] = sum[i] + cur[i] * kInv;
    }
    x.swap(sum);
  }
  ora_leaky_relu(x.data(), x.data(), x.size(), cfg->post_slope);
  const size_t ip = 1 + static_cast<size_t>(cfg->n_stages) * 19;
  ora_conv1d(x.data(), C, L, w[ip], b[ip], 1, cfg->conv_post_k, 1, round_in, wav);
  for (size_t t = 0; t < L; ++t) wav[t] = std::tanh(wav[t]);
}

// ------------------------------------------------------------------------ T2S
void ora_t2s_pe_row(int d_model, size_t pos, float* pe) {
  const size_t D = static_cast<size_t>(d_model);
  const float log_inc = static_cast<float>(-std::log(10000.0) / static_cast<double>(D));
  const float p = static_cast<float>(pos);
  for (size_t d = 0; d < D; d += 2) {
    const float div = std::exp(static_cast<float>(d) * log_inc);
    pe[d] = std::sin(p * div);
    pe[d + 1] = std::cos(p * div);
  }
}

// Attention of one head exactly as t2s_engine.cpp:1062-1087 writes it
// (KV16): scores dot_f16kv * scale over [0, n), kern::softmax over all n
// (kern.cpp:62-73: sequential max, std::exp, sequential sum, multiply by
// 1/sum), then ov += p * v (accum_f16kv) slot by slot from ov = 0.
void attend_literal(const float* q, const uint16_t* kc, const uint16_t* vc, size_t D, size_t n,
                    size_t HD, float scale, float* out) {
  std::vector<float> sc(n);
  for (size_t k = 0; k < n; ++k) sc[k] = dot_f16kv(q, kc + k * D, HD) * scale;
  ora_softmax(sc.data(), sc.data(), n);
  for (size_t e = 0; e < HD; ++e) out[e] = 0.f;
  for (size_t k = 0; k < n; ++k) accum_f16kv(out, vc + k * D, sc[k], HD);
}

// y[r] = W[r] . x with fp32 activations and widened fp16 weights in one FMA
// chain per row: the resident fp32 DenseF16 (accel.hpp:85-92) through
// sgemm at M = 1, restated in this oracle's sgemm order (ora_sgemm; the
// Accelerate kernel's own blocking is closed).
void gemv_sgemm_order(const uint16_t* w, const float* x, float* y, size_t out, size_t in) {
  row_bands(out, [&](size_t r0, size_t r1) {
    for (size_t r = r0; r < r1; ++r) y[r] = dot_f32_f16w(w + r * in, x, in);
  });
}

// T2S layers.  Every dot product uses the canonical dot32 association and
// attention the chunked softmax of attend_canon; LayerNorm is kern.cpp:27-58.
// literal != 0 instead follows t2s_engine.cpp:1036-1119 line by line where the
// canonical order departs from it: attention per attend_literal, and W2 (and,
// in ora_t2s_generate_literal, the logits head) through the fp32 DenseF16
// order of gemv_sgemm_order.
static void t2s_decode_layer(const ora_t2s_dims* dm, const ora_t2s_weights* w, int l, float* x,
                             size_t pos, uint16_t* kc, uint16_t* vc, bool literal) {
  const size_t D = dm->d_model, H = dm->n_heads, HD = D / H, F = dm->ffn;
  const size_t len = pos + 1;
  const float scale = 1.0f / std::sqrt(static_cast<float>(HD));
  std::vector<float> qkv(3 * D), attn(D), xb(D), h(D), ff(F), xr(std::max(D, F));
  // QKV on fp16(x) + bias (t2s_engine.cpp:1044-1050, GEMV16: gemv_fmlal.cpp:113)
  for (size_t i = 0; i < D; ++i) xr[i] = round_f16(x[i]);
  gemv32(w->wqkv + l * 3 * D * D, xr.data(), qkv.data(), 3 * D, D);
  for (size_t j = 0; j < 3 * D; ++j) qkv[j] = qkv[j] + w->bqkv[l * 3 * D + j];
  ora_f32_to_f16(qkv.data() + D, kc + pos * D, D);       // :1053-1055
  ora_f32_to_f16(qkv.data() + 2 * D, vc + pos * D, D);
  for (size_t hh = 0; hh < H; ++hh)  // :1062-1087
    (literal ? attend_literal : attend_canon)(qkv.data() + hh * HD, kc + hh * HD, vc + hh * HD, D,
                                              len, HD, scale, attn.data() + hh * HD);
  // out proj on fp16(attn) + bias + residual, LN1 (:1089-1099)
  for (size_t i = 0; i < D; ++i) xr[i] = round_f16(attn[i]);
  gemv32(w->wout + l * D * D, xr.data(), xb.data(), D, D);
  for (size_t i = 0; i < D; ++i) xb[i] = (xb[i] + w->bout[l * D + i]) + x[i];
  ora_layernorm(xb.data(), w->n1g + l * D, w->n1b + l * D, h.data(), D, dm->ln_eps);
  // FFN: W1 on fp16(h) + bias, ReLU; W2 on fp32 ff + bias + residual h; LN2
  for (size_t i = 0; i < D; ++i) xr[i] = round_f16(h[i]);
  gemv32(w->w1 + l * F * D, xr.data(), ff.data(), F, D);
  for (size_t i = 0; i < F; ++i) {
    const float v = ff[i] + w->b1[l * F + i];
    ff[i] = v > 0.f ? v : 0.f;
  }
  (literal ? gemv_sgemm_order : gemv32)(w->w2 + l * D * F, ff.data(), xb.data(), D, F);
  for (size_t i = 0; i < D; ++i) xb[i] = (xb[i] + w->b2[l * D + i]) + h[i];
  ora_layernorm(xb.data(), w->n2g + l * D, w->n2b + l * D, x, D, dm->ln_eps);
}

void ora_t2s_decode_layer(const ora_t2s_dims* dm, const ora_t2s_weights* w, int l, float* x,
                          size_t pos, uint16_t* kc, uint16_t* vc) {
  t2s_decode_layer(dm, w, l, x, pos, kc, vc, false);
}

void ora_t2s_decode_layer_literal(const ora_t2s_dims* dm, const ora_t2s_weights* w, int l,
                                  float* x, size_t pos, uint16_t* kc, uint16_t* vc) {
  t2s_decode_layer(dm, w, l, x, pos, kc, vc, true);
}

void ora_t2s_prefill_layer(const ora_t2s_dims* dm, const ora_t2s_weights* w, int l, float* x,
                           size_t S, size_t pos, size_t text_len, uint16_t* kc, uint16_t* vc) {
  const size_t D = dm->d_model, H = dm->n_heads, HD = D / H, F = dm->ffn;
  const float scale = 1.0f / std::sqrt(static_cast<float>(HD));
  std::vector<float> qkv(S * 3 * D), attn(S * D), tmp(S * D), ff(S * F);
  linear_canon(x, S, D, w->wqkv + l * 3 * D * D, 3 * D, w->bqkv + l * 3 * D, false, qkv.data());
  for (size_t t = 0; t < S; ++t) {
    ora_f32_to_f16(qkv.data() + t * 3 * D + D, kc + (pos + t) * D, D);
    ora_f32_to_f16(qkv.data() + t * 3 * D + 2 * D, vc + (pos + t) * D, D);
  }
  // Query q sees slots [0, pos) and block slots [0, max(text_len, q+1)):
  // the text-prefix / causal mask of t2s_engine.cpp:944-979 as one range.
  pool().run(S * H, 1, [&](size_t wb, size_t we) {
    for (size_t item = wb; item < we; ++item) {
      const size_t hh = item / S, q = item % S;
      const size_t n = pos + std::max(text_len, q + 1);
      attend_canon(qkv.data() + q * 3 * D + hh * HD, kc + hh * HD, vc + hh * HD, D, n, HD, scale,
                   attn.data() + q * D + hh * HD);
    }
  });
  linear_canon(attn.data(), S, D, w->wout + l * D * D, D, nullptr, false, tmp.data());
  for (size_t i = 0; i < S * D; ++i) x[i] = (tmp[i] + w->bout[l * D + i % D]) + x[i];
  for (size_t t = 0; t < S; ++t)
    ora_layernorm(x + t * D, w->n1g + l * D, w->n1b + l * D, x + t * D, D, dm->ln_eps);
  linear_canon(x, S, D, w->w1 + l * F * D, F, w->b1 + l * F, true, ff.data());
  linear_canon(ff.data(), S, F, w->w2 + l * D * F, D, nullptr, false, tmp.data());
  for (size_t i = 0; i < S * D; ++i) x[i] = (tmp[i] + w->b2[l * D + i % D]) + x[i];
  for (size_t t = 0; t < S; ++t)
    ora_layernorm(x + t * D, w->n2g + l * D, w->n2b + l * D, x + t * D, D, dm->ln_eps);
}

void ora_attention_decode(const float* q, const uint16_t* kc, const uint16_t* vc, size_t len,
                          size_t n_heads, size_t head_dim, size_t row_stride, float scale,
                          float* out) {
  for (size_t h = 0; h < n_heads; ++h)
    attend_canon(q + h * head_dim, kc + h * head_dim, vc + h * head_dim, row_stride, len,
                 head_dim, scale, out + h * head_dim);
}

size_t ora_hubert_front_frames(const ora_hubert_front_cfg* c, size_t n) {
  size_t t = n;
  for (int i = 0; i < 7; ++i)
    t = t < static_cast<size_t>(c->conv_kernel[i]) ? 0 : (t - c->conv_kernel[i]) / c->conv_stride[i] + 1;
  return t;
}

// hubert.cpp:476-580 (HubertEngine::run up to the transformer layers).
void ora_hubert_front(const ora_hubert_front_cfg* c, const ora_hubert_front_weights* w,
                      const float* wav, size_t n, float* out) {
  int ch = 1;
  size_t len = n;
  std::vector<float> cur(wav, wav + n), nxt;  // channel-major [ch][len]
  std::vector<uint16_t> cols;
  for (int li = 0; li < 7; ++li) {  // conv_layer, hubert.cpp:439-473
    const int k = c->conv_kernel[li], st = c->conv_stride[li], oc = c->conv_dim[li];
    const size_t T = (len - static_cast<size_t>(k)) / static_cast<size_t>(st) + 1;
    const size_t KK = static_cast<size_t>(ch) * k;
    cols.assign(T * KK, 0);
    for (size_t t = 0; t < T; ++t)
      for (int cc = 0; cc < ch; ++cc)
        for (int kk = 0; kk < k; ++kk)
          cols[t * KK + static_cast<size_t>(cc) * k + kk] = f2h(cur[static_cast<size_t>(cc) * len + t * st + kk]);
    nxt.assign(static_cast<size_t>(oc) * T, 0.f);
    ora_gemm_f16x_fmlal(w->conv_w[li], cols.data(), nxt.data(), static_cast<size_t>(oc), T, KK);
    if (li == 0) {  // GroupNorm(groups = C), hubert.cpp:485-500
      const double inv = 1.0 / static_cast<double>(T);
      for (int cc = 0; cc < oc; ++cc) {
        float* p = nxt.data() + static_cast<size_t>(cc) * T;
        double mu = 0.0, var = 0.0;
        for (size_t t = 0; t < T; ++t) mu += p[t];
        mu *= inv;
        for (size_t t = 0; t < T; ++t) var += (p[t] - mu) * (p[t] - mu);
        var *= inv;
        const double rstd = 1.0 / std::sqrt(var + c->ln_eps);
        const double g = w->gn_g[cc], b = w->gn_b[cc];
        for (size_t t = 0; t < T; ++t) p[t] = static_cast<float>((p[t] - mu) * rstd * g + b);
      }
    }
    ora_gelu_erf(nxt.data(), nxt.data(), nxt.size());
    cur.swap(nxt);
    len = T;
    ch = oc;
  }
  // feature_projection: [C6][T] -> [T][C6], LayerNorm, Linear + bias (hubert.cpp:508-529)
  const size_t T = len;
  const int C6 = c->conv_dim[6], H = c->hidden;
  std::vector<float> tmp(T * C6), x(T * H);
  for (size_t t = 0; t < T; ++t)
    for (int cc = 0; cc < C6; ++cc) tmp[t * C6 + cc] = cur[static_cast<size_t>(cc) * T + t];
  for (size_t t = 0; t < T; ++t)
    ora_layernorm(tmp.data() + t * C6, w->proj_ln_g, w->proj_ln_b, tmp.data() + t * C6, C6, c->ln_eps);
  ora_linear_f16(tmp.data(), T, C6, w->proj_w, H, w->proj_b, ORA_ACT_NONE, 0.f, x.data());
  // pos_conv (hubert.cpp:531-577): grouped conv, pad K/2, T + 1 outputs, + bias,
  // GELU, SamePad drops the last frame, x += it
  const int G = c->pos_groups, cg = H / G, K = c->pos_k;
  const size_t P = static_cast<size_t>(K) / 2, Tp = T + 1, KK = static_cast<size_t>(cg) * K;
  std::vector<uint16_t> w16(static_cast<size_t>(H) * cg * K);
  ora_f32_to_f16(w->pos_w, w16.data(), w16.size());
  std::vector<float> pos(Tp * H), gt(static_cast<size_t>(cg) * Tp);
  cols.assign(Tp * KK, 0);
  for (int g = 0; g < G; ++g) {
    for (size_t t = 0; t < Tp; ++t)
      for (int j = 0; j < cg; ++j)
        for (int kk = 0; kk < K; ++kk) {
          const size_t src = t + kk;
          const float v = (src >= P && src < P + T) ? x[(src - P) * H + static_cast<size_t>(g) * cg + j] : 0.f;
          cols[t * KK + static_cast<size_t>(j) * K + kk] = f2h(v);
        }
    ora_gemm_f16x_fmlal(w16.data() + static_cast<size_t>(g) * cg * KK, cols.data(), gt.data(),
                        static_cast<size_t>(cg), Tp, KK);
    for (size_t t = 0; t < Tp; ++t)
      for (int i = 0; i < cg; ++i)
        pos[t * H + static_cast<size_t>(g) * cg + i] = gt[static_cast<size_t>(i) * Tp + t];
  }
  for (size_t t = 0; t < Tp; ++t)
    for (int i = 0; i < H; ++i) pos[t * H + i] = pos[t * H + i] + w->pos_b[i];
  ora_gelu_erf(pos.data(), pos.data(), pos.size());
  for (size_t t = 0; t < T; ++t)
    for (int i = 0; i < H; ++i) x[t * H + i] = x[t * H + i] + pos[t * H + i];
  for (size_t t = 0; t < T; ++t)  // encoder.layer_norm
    ora_layernorm(x.data() + t * H, w->enc_ln_g, w->enc_ln_b, out + t * H, H, c->ln_eps);
}

// bert_ops.hpp:347-400 BertLayer::forward (and the HuBERT layer loop,
// hubert.cpp:590-730, which has the same post-LN structure): q/k/v via the
// DenseF16 view (fp16 activations, fp32 accumulation) + bias; per head
// S = (Q K^T) / sqrt(dh) (+ key mask), softmax rows, ctx = S V in fp32;
// attn_out + bias + residual, LN; inter + bias, GELU(erf); ffn_out + bias +
// residual, LN.  x [B*T][C] in place; valid (optional) holds the number of
// real tokens per utterance (mask value finfo.min on the rest, :373-374).
void ora_encoder_layer(const ora_encoder_dims* d, const ora_encoder_weights* w, int l, float* x,
                       int B, int T, const int* valid) {
  const size_t C = d->hidden, H = d->heads, dh = C / H, F = d->ffn, M = (size_t)B * T;
  std::vector<float> q(M * C), k(M * C), v(M * C), ctx(M * C), y(M * C), mid(M * F), f2(M * C);
  const size_t oqkv = (size_t)l * 3 * C * C, ob = (size_t)l * 3 * C;
  ora_linear_f16(x, M, C, w->wqkv + oqkv, C, w->bqkv + ob, ORA_ACT_NONE, 0.f, q.data());
  ora_linear_f16(x, M, C, w->wqkv + oqkv + C * C, C, w->bqkv + ob + C, ORA_ACT_NONE, 0.f, k.data());
  ora_linear_f16(x, M, C, w->wqkv + oqkv + 2 * C * C, C, w->bqkv + ob + 2 * C, ORA_ACT_NONE, 0.f,
                 v.data());
  const float alpha = 1.f / std::sqrt(static_cast<float>(dh));
  pool().run((size_t)B * H, 1, [&](size_t ib, size_t ie) {
    std::vector<float> S((size_t)T * T);
    for (size_t item = ib; item < ie; ++item) {
      const size_t b = item / H, h = item % H;
      const int nv = valid ? valid[b] : T;
      for (int i = 0; i < T; ++i)
        for (int j = 0; j < T; ++j) {
          float acc = 0.f;
          const float* qi = q.data() + ((b * T + i) * C + h * dh);
          const float* kj = k.data() + ((b * T + j) * C + h * dh);
          for (size_t e = 0; e < dh; ++e) acc = std::fmaf(qi[e], kj[e], acc);
          float s = alpha * acc;
          if (j >= nv) s = s + -3.40282347e+38f;
          S[(size_t)i * T + j] = s;
        }
      for (int i = 0; i < T; ++i) {  // bert_ops.hpp:28-43 softmax_rows
        float* r = S.data() + (size_t)i * T;
        float mx = r[0];
        for (int j = 1; j < T; ++j) mx = mx > r[j] ? mx : r[j];
        float sum = 0.f;
        for (int j = 0; j < T; ++j) {
          r[j] = std::exp(r[j] - mx);
          sum = sum + r[j];
        }
        const float inv = 1.f / sum;
        for (int j = 0; j < T; ++j) r[j] = r[j] * inv;
      }
      for (int i = 0; i < T; ++i)
        for (size_t e = 0; e < dh; ++e) {
          float acc = 0.f;
          for (int j = 0; j < T; ++j)
            acc = std::fmaf(S[(size_t)i * T + j], v[(b * T + j) * C + h * dh + e], acc);
          ctx[(b * T + i) * C + h * dh + e] = acc;
        }
    }
  });
  ora_linear_f16(ctx.data(), M, C, w->wo + (size_t)l * C * C, C, w->bo + (size_t)l * C,
                 ORA_ACT_NONE, 0.f, y.data());
  for (size_t i = 0; i < M * C; ++i) y[i] = y[i] + x[i];
  for (size_t r = 0; r < M; ++r)
    ora_layernorm(y.data() + r * C, w->ln1g + (size_t)l * C, w->ln1b + (size_t)l * C,
                  y.data() + r * C, C, d->eps);
  ora_linear_f16(y.data(), M, C, w->wi + (size_t)l * F * C, F, w->bi + (size_t)l * F,
                 ORA_ACT_GELU_ERF, 0.f, mid.data());
  ora_linear_f16(mid.data(), M, F, w->wf + (size_t)l * C * F, C, w->bf + (size_t)l * C,
                 ORA_ACT_NONE, 0.f, f2.data());
  for (size_t i = 0; i < M * C; ++i) f2[i] = f2[i] + y[i];
  for (size_t r = 0; r < M; ++r)
    ora_layernorm(f2.data() + r * C, w->ln2g + (size_t)l * C, w->ln2b + (size_t)l * C,
                  x + r * C, C, d->eps);
}

int ora_t2s_greedy_sample(float* lg, int V, const int32_t* hist, size_t n_hist,
                          int eos_allowed, int* raw_argmax) {
  const int limit = eos_allowed ? V : V - 1;
  std::vector<unsigned char> mark(static_cast<size_t>(V), 0);
  for (size_t i = 0; i < n_hist; ++i) {
    const int c = hist[i];
    if (c < 0 || c >= limit || mark[c]) continue;
    mark[c] = 1;
    float& v = lg[c];
    v = v < 0.f ? v * 1.35f : v / 1.35f;
  }
  if (raw_argmax) {
    int best = 0;
    float bv = lg[0];
    for (int c = 1; c < V; ++c)
      if (lg[c] > bv) {
        bv = lg[c];
        best = c;
      }
    *raw_argmax = best;
  }
  int best = 0;
  float bv = lg[0];
  for (int c = 1; c < limit; ++c)
    if (lg[c] > bv) {
      bv = lg[c];
      best = c;
    }
  return best;
}

// t2s_engine.cpp:1640-1737 topk_sample: repetition penalty (once per distinct
// history token below `limit`), top-k by the reference's selection sort
// (strict '>' over the current positions, swapping into place), temperature,
// softmax over the k values (exp_det in place of libm expf, as in the
// canonical attention), top-p from the tail, then a multinomial draw
// u = uniform(rng) * sum: uniform_real_distribution<float>(0, 1) on
// std::mt19937_64, which the reference's libc++ evaluates as one 64-bit draw
// converted to float and scaled by 2^-64 (generate_canonical<float, 24>).
// Returns the sampled token; *margin receives top1 - top2 of the penalised
// logits over [0, limit).
static int ora_t2s_topk_sample(float* lg, int V, const int32_t* hist, size_t n_hist, int eos_allowed,
                               const ora_sampling* sp, std::mt19937_64* rng, float* margin) {
  const int limit = eos_allowed ? V : V - 1;
  std::vector<unsigned char> mark(static_cast<size_t>(V), 0);
  for (size_t i = 0; i < n_hist; ++i) {
    const int c = hist[i];
    if (c < 0 || c >= limit || mark[c]) continue;
    mark[c] = 1;
    float& v = lg[c];
    v = v < 0.f ? v * sp->rep_penalty : v / sp->rep_penalty;
  }
  if (margin) {
    float b = -INFINITY, s2 = -INFINITY;
    int bi = -1;
    for (int c = 0; c < limit; ++c)
      if (lg[c] > b) {
        b = lg[c];
        bi = c;
      }
    for (int c = 0; c < limit; ++c)
      if (c != bi && lg[c] > s2) s2 = lg[c];
    *margin = b - s2;
  }
  const int k = sp->top_k > limit ? limit : (sp->top_k < 1 ? 1 : sp->top_k);
  std::vector<int> idxs(static_cast<size_t>(limit));
  std::vector<float> vals(static_cast<size_t>(limit));
  for (int c = 0; c < limit; ++c) {
    idxs[c] = c;
    vals[c] = lg[c];
  }
  for (int i = 0; i < k; ++i) {
    int max_j = i;
    float max_v = vals[i];
    for (int j = i + 1; j < limit; ++j)
      if (vals[j] > max_v) {
        max_v = vals[j];
        max_j = j;
      }
    if (max_j != i) {
      std::swap(vals[i], vals[max_j]);
      std::swap(idxs[i], idxs[max_j]);
    }
  }
  if (sp->temperature <= 0.f) {
    int best = idxs[0];
    float bv = vals[0];
    for (int i = 1; i < k; ++i)
      if (vals[i] > bv) {
        bv = vals[i];
        best = idxs[i];
      }
    return best;
  }
  if (sp->temperature != 1.0f)
    for (int i = 0; i < k; ++i) vals[i] = vals[i] / sp->temperature;
  float max_logit = vals[0];
  for (int i = 1; i < k; ++i)
    if (vals[i] > max_logit) max_logit = vals[i];
  float sum_exp = 0.f;
  for (int i = 0; i < k; ++i) {
    vals[i] = exp_det(vals[i] - max_logit);
    sum_exp = sum_exp + vals[i];
  }
  int keep = k;
  if (sp->top_p < 1.0f) {
    const float threshold = (1.f - sp->top_p) * sum_exp;
    float cum = 0.f;
    for (int i = k - 1; i >= 0; --i) {
      cum = cum + vals[i];
      if (cum >= threshold) {
        keep = i + 1;
        break;
      }
    }
    if (keep < k) {
      sum_exp = 0.f;
      for (int i = 0; i < keep; ++i) sum_exp = sum_exp + vals[i];
    }
  }
  const float u01 = static_cast<float>((*rng)()) * 0x1p-64f;
  const float u = u01 * sum_exp;
  float cdf = 0.f;
  for (int i = 0; i < keep; ++i) {
    cdf = cdf + vals[i];
    if (u <= cdf) return idxs[i];
  }
  return idxs[keep - 1];
}

static int t2s_generate(const ora_t2s_dims* dm, const ora_t2s_weights* w, uint16_t* kc,
                        uint16_t* vc, size_t cap, size_t prefix, const int32_t* prompt, size_t P,
                        size_t max_steps, int stop_on_eos, int32_t* tokens_out,
                        float* margins_out, float* last_logits, float* all_logits, bool literal,
                        const ora_sampling* sp = nullptr) {
  const bool topk = sp && sp->mode == 1;
  std::mt19937_64 rng(sp ? sp->seed : 0);  // t2s_engine.cpp:1814-1818
  auto logits_head = literal ? gemv_sgemm_order : gemv32;  // predict_layer_fp, :704-708
  const size_t D = dm->d_model, L = dm->n_layers, V = dm->vocab;
  const int eos = static_cast<int>(V) - 1;
  if (P == 0 || prefix + P + max_steps > cap) return -1;
  std::vector<float> xy(P * D), pe(D), x1(D), logits(V);
  for (size_t t = 0; t < P; ++t) {  // t2s_engine.cpp:1785-1790
    ora_t2s_pe_row(dm->d_model, t, pe.data());
    const uint16_t* er = w->audio_emb + static_cast<size_t>(prompt[t]) * D;
    for (size_t d = 0; d < D; ++d) xy[t * D + d] = std::fmaf(dm->alpha_audio, pe[d], h2f(er[d]));
  }
  for (size_t l = 0; l < L; ++l)
    ora_t2s_prefill_layer(dm, w, static_cast<int>(l), xy.data(), P, prefix, 0, kc + l * cap * D,
                          vc + l * cap * D);
  logits_head(w->wpred, xy.data() + (P - 1) * D, logits.data(), V, D);  // fp32 activations
  std::vector<int32_t> hist(prompt, prompt + P);
  size_t cur = prefix + P;
  int n_out = 0;
  for (size_t idx = 0; idx < max_steps; ++idx) {
    const bool eos_allowed = idx >= 11;  // kEosMaskSteps
    if (last_logits) std::memcpy(last_logits, logits.data(), V * sizeof(float));
    if (all_logits) std::memcpy(all_logits + idx * V, logits.data(), V * sizeof(float));
    int raw = -1;
    float tk_margin = 0.f;
    const int s = topk ? ora_t2s_topk_sample(logits.data(), static_cast<int>(V), hist.data(),
                                             hist.size(), eos_allowed, sp, &rng, &tk_margin)
                       : ora_t2s_greedy_sample(logits.data(), static_cast<int>(V), hist.data(),
                                               hist.size(), eos_allowed, &raw);
    if (topk && margins_out) margins_out[idx] = tk_margin;
    if (!topk && margins_out) {
      const int limit = eos_allowed ? static_cast<int>(V) : static_cast<int>(V) - 1;
      float second = -INFINITY;
      for (int c = 0; c < limit; ++c)
        if (c != s && logits[c] > second) second = logits[c];
      margins_out[idx] = logits[s] - second;
    }
    bool stop = false;
    if (stop_on_eos && eos_allowed && s == eos) {
      stop = true;
    } else {
      tokens_out[n_out++] = s;
      hist.push_back(s);
    }
    if (idx + 1 == max_steps) stop = true;
    if (stop) break;
    ora_t2s_pe_row(dm->d_model, P + idx, pe.data());  // :1865-1869
    const uint16_t* er = w->audio_emb + static_cast<size_t>(s) * D;
    for (size_t d = 0; d < D; ++d) x1[d] = std::fmaf(dm->alpha_audio, pe[d], h2f(er[d]));
    for (size_t l = 0; l < L; ++l)
      t2s_decode_layer(dm, w, static_cast<int>(l), x1.data(), cur, kc + l * cap * D,
                       vc + l * cap * D, literal);
    logits_head(w->wpred, x1.data(), logits.data(), V, D);
    ++cur;
  }
  return n_out;
}

int ora_t2s_generate(const ora_t2s_dims* dm, const ora_t2s_weights* w, uint16_t* kc,
                     uint16_t* vc, size_t cap, size_t prefix, const int32_t* prompt, size_t P,
                     size_t max_steps, int stop_on_eos, int32_t* tokens_out,
                     float* margins_out, float* last_logits) {
  return t2s_generate(dm, w, kc, vc, cap, prefix, prompt, P, max_steps, stop_on_eos, tokens_out,
                      margins_out, last_logits, nullptr, false);
}

int ora_t2s_generate_sampled(const ora_t2s_dims* dm, const ora_t2s_weights* w, uint16_t* kc,
                             uint16_t* vc, size_t cap, size_t prefix, const int32_t* prompt,
                             size_t P, size_t max_steps, int stop_on_eos, const ora_sampling* sp,
                             int32_t* tokens_out, float* margins_out) {
  return t2s_generate(dm, w, kc, vc, cap, prefix, prompt, P, max_steps, stop_on_eos, tokens_out,
                      margins_out, nullptr, nullptr, false, sp);
}

int ora_t2s_generate_ex(const ora_t2s_dims* dm, const ora_t2s_weights* w, uint16_t* kc,
                        uint16_t* vc, size_t cap, size_t prefix, const int32_t* prompt, size_t P,
                        size_t max_steps, int stop_on_eos, int literal, int32_t* tokens_out,
                        float* margins_out, float* all_logits) {
  return t2s_generate(dm, w, kc, vc, cap, prefix, prompt, P, max_steps, stop_on_eos, tokens_out,
                      margins_out, nullptr, all_logits, literal != 0);
}

}  // extern "C"

// ------------------------------------------------------- SoVITS latent path
// sovits_engine.hpp:48-93 steps 1-5, channel-major [C][T] as the reference's
// Tensor2D (sovits_types.hpp:21-35).
namespace {

struct LatentError {
  int code;
};

class Named {
 public:
  Named(const ora_named* t, size_t n) {
    for (size_t i = 0; i < n; ++i) by_[t[i].name] = &t[i];
  }
  bool has(const std::string& n) const { return by_.count(n) != 0; }
  const ora_named& get(const std::string& n, uint64_t numel) const {
    auto it = by_.find(n);
    if (it == by_.end() || (numel && it->second->numel != numel) ||
        (!it->second->f32 && !it->second->f16))
      throw LatentError{-1};
    return *it->second;
  }
  // load_tensor_f32 (sovits_types.hpp:38-48): the fp16 copy, widened, when
  // the file holds one; else the fp32 copy.
  std::vector<float> f32(const std::string& n, uint64_t numel = 0) const {
    const ora_named& t = get(n, numel);
    std::vector<float> v(t.numel);
    if (t.f16)
      ora_f16_to_f32(t.f16, v.data(), t.numel);
    else
      std::copy(t.f32, t.f32 + t.numel, v.begin());
    return v;
  }
  // load_tensor_f16 (sovits_types.hpp:76-87): the fp16 copy, else the fp32
  // copy rounded once.
  std::vector<uint16_t> f16(const std::string& n, uint64_t numel = 0) const {
    const ora_named& t = get(n, numel);
    std::vector<uint16_t> v(t.numel);
    if (t.f16)
      std::copy(t.f16, t.f16 + t.numel, v.begin());
    else
      ora_f32_to_f16(t.f32, v.data(), t.numel);
    return v;
  }

 private:
  std::map<std::string, const ora_named*> by_;
};

using Vec = std::vector<float>;

// sovits::Conv1d (conv1d.hpp:57-82, forward :109-194).
struct LConv {
  size_t co = 0, ci = 0, k = 1;
  std::vector<uint16_t> w;
  Vec b;
  void load(const Named& T, const std::string& p, size_t o, size_t i, size_t kk) {
    co = o, ci = i, k = kk;
    w = T.f16(p + ".weight", o * i * kk);
    b = T.has(p + ".bias") ? T.f32(p + ".bias", o) : Vec(o, 0.f);
  }
  Vec operator()(const Vec& x, size_t T, bool round_in = true) const {
    Vec y(co * T);
    ora_conv1d(x.data(), ci, T, w.data(), b.data(), co, k, 1, round_in ? 1 : 0, y.data());
    return y;
  }
};

// sovits::MultiHeadAttention (mha.hpp:16-202) with an all-ones mask.
struct LMha {
  size_t C = 0, H = 0, dk = 0, table = 0;
  LConv q, k, v, o;
  Vec relk, relv;
  void load(const Named& T, const std::string& p, size_t ch, size_t heads, size_t tab) {
    C = ch, H = heads, dk = ch / heads, table = tab;
    q.load(T, p + ".conv_q", ch, ch, 1);
    k.load(T, p + ".conv_k", ch, ch, 1);
    v.load(T, p + ".conv_v", ch, ch, 1);
    o.load(T, p + ".conv_o", ch, ch, 1);
    if (tab) {
      relk = T.f32(p + ".emb_rel_k", tab * dk);
      relv = T.f32(p + ".emb_rel_v", tab * dk);
    }
  }
  // _get_relative_embeddings (mha.hpp:45-58).
  Vec slice(const Vec& emb, size_t L) const {
    const size_t hw = table / 2;
    const size_t pad_len = L > hw + 1 ? L - (hw + 1) : 0;
    const size_t start = hw + 1 > L ? hw + 1 - L : 0;
    Vec used((2 * L - 1) * dk, 0.f);
    for (size_t m = 0; m < 2 * L - 1; ++m) {
      const long long src = static_cast<long long>(m + start) - static_cast<long long>(pad_len);
      if (src >= 0 && src < static_cast<long long>(table))
        for (size_t d = 0; d < dk; ++d) used[m * dk + d] = emb[src * dk + d];
    }
    return used;
  }
  Vec operator()(const Vec& xq, size_t Tq, const Vec& xkv, size_t Tk) const {
    const Vec qb = q(xq, Tq), kb = k(xkv, Tk), vb = v(xkv, Tk);
    const float scale = 1.f / std::sqrt(static_cast<float>(dk));
    Vec sc(H * Tq * Tk);
    Vec usedk, usedv, rl;
    const size_t L = Tq;
    if (table) {
      usedk = slice(relk, L);
      usedv = slice(relv, L);
      rl.assign(H * L * (2 * L - 1), 0.f);
    }
    pool().run(H * Tq, 1, [&](size_t rb, size_t re) {
      for (size_t r = rb; r < re; ++r) {
        const size_t h = r / Tq, i = r % Tq;
        // scores = scale * Q[h]^T K[h] (mha.hpp:80-90, an sgemm with alpha)
        for (size_t j = 0; j < Tk; ++j) {
          float acc = 0.f;
          for (size_t d = 0; d < dk; ++d)
            acc = std::fmaf(qb[(h * dk + d) * Tq + i], kb[(h * dk + d) * Tk + j], acc);
          sc[(h * Tq + i) * Tk + j] = scale * acc;
        }
        if (table)  // rel_logits = scale * Q[h]^T usedk^T (mha.hpp:105-113)
          for (size_t m = 0; m < 2 * L - 1; ++m) {
            float acc = 0.f;
            for (size_t d = 0; d < dk; ++d)
              acc = std::fmaf(qb[(h * dk + d) * Tq + i], usedk[m * dk + d], acc);
            rl[(h * L + i) * (2 * L - 1) + m] = scale * acc;
          }
      }
    });
    if (table)  // relative -> absolute (mha.hpp:122-135)
      for (size_t h = 0; h < H; ++h)
        for (size_t i = 0; i < L; ++i)
          for (size_t j = 0; j < L; ++j) {
            const size_t nn = i * (2 * L - 1) + j + L - 1;
            float val = 0.f;
            if (nn < 2 * L * L) {
              const size_t a = nn / (2 * L), bb = nn % (2 * L);
              if (bb != 2 * L - 1) val = rl[(h * L + a) * (2 * L - 1) + bb];
            }
            sc[(h * L + i) * Tk + j] += val;
          }
    // softmax_row_inplace (nn_ops.hpp:12-22)
    for (size_t r = 0; r < H * Tq; ++r) {
      float* x = &sc[r * Tk];
      float mx = x[0];
      for (size_t s = 1; s < Tk; ++s) mx = std::max(mx, x[s]);
      float sum = 0.f;
      for (size_t s = 0; s < Tk; ++s) {
        x[s] = std::exp(x[s] - mx);
        sum += x[s];
      }
      const float inv = 1.f / sum;
      for (size_t s = 0; s < Tk; ++s) x[s] *= inv;
    }
    // out = sum_s p v (mha.hpp:164-175), then the relative values (:176-196)
    Vec out(C * Tq, 0.f);
    for (size_t h = 0; h < H; ++h)
      for (size_t t = 0; t < Tq; ++t) {
        const float* pr = &sc[(h * Tq + t) * Tk];
        for (size_t s = 0; s < Tk; ++s) {
          const float p = pr[s];
          if (p == 0.f) continue;
          for (size_t d = 0; d < dk; ++d)
            out[(h * dk + d) * Tq + t] += p * vb[(h * dk + d) * Tk + s];
        }
      }
    if (table)
      for (size_t h = 0; h < H; ++h)
        for (size_t i = 0; i < L; ++i)
          for (size_t m = 0; m < 2 * L - 1; ++m) {
            const size_t nn = i * 2 * L + m + 1;
            float w = 0.f;
            if (nn >= L) {
              const size_t mm = nn - L;
              const size_t a = mm / (2 * L - 1), bb = mm % (2 * L - 1);
              w = bb < L ? sc[(h * L + a) * L + bb] : 0.f;
            }
            if (w == 0.f) continue;
            for (size_t d = 0; d < dk; ++d) out[(h * dk + d) * Tq + i] += w * usedv[m * dk + d];
          }
    return o(out, Tq);
  }
};

// layernorm_ct (nn_ops.hpp:26-45): per frame over the channels, eps 1e-5.
Vec layernorm_ct(const Vec& x, const Vec& g, const Vec& b, size_t C, size_t T) {
  Vec y(C * T);
  for (size_t t = 0; t < T; ++t) {
    float mu = 0.f;
    for (size_t c = 0; c < C; ++c) mu += x[c * T + t];
    mu /= static_cast<float>(C);
    float var = 0.f;
    for (size_t c = 0; c < C; ++c) {
      const float d = x[c * T + t] - mu;
      var += d * d;
    }
    var /= static_cast<float>(C);
    const float inv = 1.f / std::sqrt(var + 1e-5f);
    for (size_t c = 0; c < C; ++c) y[c * T + t] = (x[c * T + t] - mu) * inv * g[c] + b[c];
  }
  return y;
}

// sovits::Encoder (enc_p_parts.hpp:34-95): rel-MHA, LN, FFN(k, ReLU), LN.
struct LEncoder {
  struct Layer {
    LMha attn;
    Vec g1, b1, g2, b2;
    LConv f1, f2;
  };
  size_t C = 0;
  std::vector<Layer> layers;
  void load(const Named& T, const std::string& p, size_t ch, size_t heads, size_t nl,
            size_t filt, size_t k, size_t table) {
    C = ch;
    layers.resize(nl);
    for (size_t i = 0; i < nl; ++i) {
      const std::string ix = "." + std::to_string(i);
      Layer& L = layers[i];
      L.attn.load(T, p + ".attn_layers" + ix, ch, heads, table);
      L.g1 = T.f32(p + ".norm_layers_1" + ix + ".gamma", ch);
      L.b1 = T.f32(p + ".norm_layers_1" + ix + ".beta", ch);
      L.g2 = T.f32(p + ".norm_layers_2" + ix + ".gamma", ch);
      L.b2 = T.f32(p + ".norm_layers_2" + ix + ".beta", ch);
      L.f1.load(T, p + ".ffn_layers" + ix + ".conv_1", filt, ch, k);
      L.f2.load(T, p + ".ffn_layers" + ix + ".conv_2", ch, filt, k);
    }
  }
  void forward(Vec& x, size_t T) const {
    Vec s(C * T);
    for (const Layer& L : layers) {
      const Vec y = L.attn(x, T, x, T);
      for (size_t i = 0; i < C * T; ++i) s[i] = x[i] + y[i];
      x = layernorm_ct(s, L.g1, L.b1, C, T);
      Vec h = L.f1(x, T);
      for (float& v : h) v = v > 0.f ? v : 0.f;
      const Vec f = L.f2(h, T);
      for (size_t i = 0; i < C * T; ++i) s[i] = x[i] + f[i];
      x = layernorm_ct(s, L.g2, L.b2, C, T);
    }
  }
};

int sovits_latent(const ora_sovits_latent_cfg* c, const Named& N, const int64_t* codes, size_t Tc,
                  const int64_t* phones, size_t Tt, const float* ge, const float* ge_text,
                  const float* noise, float* m_p_out, float* logs_p_out, float* z_out) {
  const size_t D = c->ssl_dim, C = c->hidden, Tq = 2 * Tc, half = C / 2, nl = c->wn_layers;
  const size_t table = 2 * c->window + 1, MH = c->mrte_hidden;
  // 1-2. RVQ decode (quantizer.hpp:26-38) and nearest x2 (sovits_engine.hpp:57-64)
  const ora_named& cb = N.get("quantizer.vq.layers.0._codebook.embed", 0);
  const Vec embed = N.f32(cb.name);
  const size_t n_codes = embed.size() / D;
  Vec up(D * Tq);
  for (size_t t = 0; t < Tc; ++t) {
    if (codes[t] < 0 || static_cast<size_t>(codes[t]) >= n_codes) throw LatentError{-2};
    for (size_t d = 0; d < D; ++d)
      up[d * Tq + 2 * t] = up[d * Tq + 2 * t + 1] = embed[codes[t] * D + d];
  }
  // 3. TextEncoder (enc_p.hpp:45-91)
  LConv ssl_proj, c_pre, text_pre, c_post, proj;
  ssl_proj.load(N, "enc_p.ssl_proj", C, D, 1);
  LEncoder e_ssl, e_text, e2;
  e_ssl.load(N, "enc_p.encoder_ssl", C, c->heads, c->layers_ssl, c->filter, c->kernel, table);
  e_text.load(N, "enc_p.encoder_text", C, c->heads, c->layers_text, c->filter, c->kernel, table);
  e2.load(N, "enc_p.encoder2", C, c->heads, c->layers_2, c->filter, c->kernel, table);
  const Vec temb_w = N.f32("enc_p.text_embedding.weight");
  const size_t n_sym = temb_w.size() / C;
  LMha cross;
  cross.load(N, "enc_p.mrte.cross_attention", MH, c->mrte_heads, 0);
  c_pre.load(N, "enc_p.mrte.c_pre", MH, C, 1);
  text_pre.load(N, "enc_p.mrte.text_pre", MH, C, 1);
  c_post.load(N, "enc_p.mrte.c_post", C, MH, 1);
  proj.load(N, "enc_p.proj", 2 * C, C, 1);

  Vec y = ssl_proj(up, Tq);
  e_ssl.forward(y, Tq);
  Vec temb(C * Tt);
  for (size_t t = 0; t < Tt; ++t) {
    if (phones[t] < 0 || static_cast<size_t>(phones[t]) >= n_sym) throw LatentError{-2};
    for (size_t ch = 0; ch < C; ++ch) temb[ch * Tt + t] = temb_w[phones[t] * C + ch];
  }
  e_text.forward(temb, Tt);
  // MRTE (enc_p_parts.hpp:111-129)
  const Vec c512 = c_pre(y, Tq), t512 = text_pre(temb, Tt);
  const Vec att = cross(c512, Tq, t512, Tt);
  Vec sum(MH * Tq);
  for (size_t ch = 0; ch < MH; ++ch)
    for (size_t t = 0; t < Tq; ++t)
      sum[ch * Tq + t] = att[ch * Tq + t] + c512[ch * Tq + t] + ge_text[ch];
  Vec m = c_post(sum, Tq);
  e2.forward(m, Tq);
  const Vec stats = proj(m, Tq);
  // 4. z_p = m_p + noise * exp(logs_p) * noise_scale (sovits_engine.hpp:74-79)
  Vec x(C * Tq);
  for (size_t i = 0; i < C * Tq; ++i) {
    const float mp = stats[i], lp = stats[C * Tq + i];
    if (m_p_out) m_p_out[i] = mp;
    if (logs_p_out) logs_p_out[i] = lp;
    x[i] = mp + (noise ? noise[i] : 0.f) * std::exp(lp) * c->noise_scale;
  }
  // 5. reverse flow (flow.hpp:136-170): flip, then the coupling layer
  const Vec gev(ge, ge + c->gin);
  for (int f = c->flows - 1; f >= 0; --f) {
    for (size_t ch = 0; ch < C / 2; ++ch)
      for (size_t t = 0; t < Tq; ++t) std::swap(x[ch * Tq + t], x[(C - 1 - ch) * Tq + t]);
    const std::string p = "flow.flows." + std::to_string(2 * f);
    LConv pre, cond, post;
    pre.load(N, p + ".pre", C, half, 1);
    cond.load(N, p + ".enc.cond_layer", 2 * C * nl, c->gin, 1);
    post.load(N, p + ".post", half, C, 1);
    const Vec x0(x.begin(), x.begin() + half * Tq);
    Vec h = pre(x0, Tq);
    // FlowWN::forward (flow.hpp:38-106); the cond layer sees one frame and
    // takes the fp32 path
    const Vec g = cond(gev, 1, false);
    Vec out(C * Tq, 0.f), acts(C * Tq);
    for (size_t l = 0; l < nl; ++l) {
      LConv in, rs;
      in.load(N, p + ".enc.in_layers." + std::to_string(l), 2 * C, C, c->wn_kernel);
      rs.load(N, p + ".enc.res_skip_layers." + std::to_string(l), l + 1 < nl ? 2 * C : C, C, 1);
      const Vec a = in(h, Tq);
      for (size_t ch = 0; ch < C; ++ch)
        for (size_t t = 0; t < Tq; ++t)
          acts[ch * Tq + t] =
              std::tanh(a[ch * Tq + t] + g[l * 2 * C + ch]) *
              (1.f / (1.f + std::exp(-(a[(C + ch) * Tq + t] + g[l * 2 * C + C + ch]))));
      const Vec r = rs(acts, Tq);
      if (l + 1 < nl) {
        for (size_t i = 0; i < C * Tq; ++i) h[i] = (h[i] + r[i]) * 1.f;
        for (size_t i = 0; i < C * Tq; ++i) out[i] += r[C * Tq + i];
      } else {
        for (size_t i = 0; i < C * Tq; ++i) out[i] += r[i];
      }
    }
    const Vec mm = post(out, Tq);
    for (size_t i = 0; i < half * Tq; ++i) x[half * Tq + i] -= mm[i];
  }
  std::copy(x.begin(), x.end(), z_out);
  return 0;
}

}  // namespace

extern "C" int ora_sovits_latent(const ora_sovits_latent_cfg* c, const ora_named* t, size_t n,
                                 const int64_t* codes, size_t Tc, const int64_t* phones,
                                 size_t Tt, const float* ge, const float* ge_text,
                                 const float* noise, float* m_p, float* logs_p, float* z) {
  try {
    const Named N(t, n);
    return sovits_latent(c, N, codes, Tc, phones, Tt, ge, ge_text, noise, m_p, logs_p, z);
  } catch (const LatentError& e) {
    return e.code;
  }
}

// ------------------------------------------------- SV speaker encoder
// sv.cpp:130-885 (the default, non --amx-enc path), channel-major
// [C][H][W] like the reference.
namespace {

struct SvMissing {};

const ora_named* sv_find(const std::map<std::string, const ora_named*>& by, const std::string& n) {
  auto it = by.find(n);
  return it == by.end() ? nullptr : it->second;
}

// vec_any (sv.cpp:74-84): the fp16 copy widened when present, else fp32.
std::vector<float> sv_vec(const std::map<std::string, const ora_named*>& by, const std::string& n) {
  const ora_named* t = sv_find(by, n);
  if (!t || (!t->f16 && !t->f32)) throw SvMissing{};
  std::vector<float> v(t->numel);
  if (t->f16)
    ora_f16_to_f32(t->f16, v.data(), t->numel);
  else
    std::copy(t->f32, t->f32 + t->numel, v.begin());
  return v;
}

// load_conv_w (sv.cpp:97-128): the fp16 copy, else the fp32 copy rounded.
std::vector<uint16_t> sv_w16(const std::map<std::string, const ora_named*>& by,
                             const std::string& n) {
  const ora_named* t = sv_find(by, n);
  if (!t || (!t->f16 && !t->f32)) throw SvMissing{};
  std::vector<uint16_t> v(t->numel);
  if (t->f16)
    std::copy(t->f16, t->f16 + t->numel, v.begin());
  else
    ora_f32_to_f16(t->f32, v.data(), t->numel);
  return v;
}

struct SvBn {
  std::vector<float> g, b, mean, var;
  void load(const std::map<std::string, const ora_named*>& by, const std::string& p) {
    g = sv_vec(by, p + ".weight");
    b = sv_vec(by, p + ".bias");
    mean = sv_vec(by, p + ".running_mean");
    var = sv_vec(by, p + ".running_var");
  }
  // Bn::apply (sv.cpp:132-145), the fp64 chain.
  void apply(float* x, int c, size_t s) const {
    for (int ci = 0; ci < c; ++ci) {
      const double a0 = static_cast<double>(g[ci]) / std::sqrt(static_cast<double>(var[ci]) + 1e-5);
      const double beta0 = static_cast<double>(b[ci]), mu0 = static_cast<double>(mean[ci]);
      float* row = x + static_cast<size_t>(ci) * s;
      for (size_t i = 0; i < s; ++i)
        row[i] = static_cast<float>((static_cast<double>(row[i]) - mu0) * a0 + beta0);
    }
  }
};

inline float relu20f(float v) { return v < 0.f ? 0.f : (v > 20.f ? 20.f : v); }

// conv2d (sv.cpp:171-194): im2col in fp32, sgemm('N','T').
std::vector<float> sv_conv2d_f32(const float* in, int c_in, int h, int w, const float* wt,
                                 int c_out, int kh, int kw, int stride, int pad) {
  const int oh = (h + 2 * pad - kh) / stride + 1, ow = (w + 2 * pad - kw) / stride + 1;
  const size_t S = static_cast<size_t>(oh) * ow;
  const int K = c_in * kh * kw;
  std::vector<float> cols(S * K);
  for (int oy = 0; oy < oh; ++oy)
    for (int ox = 0; ox < ow; ++ox) {
      float* row = cols.data() + (static_cast<size_t>(oy) * ow + ox) * K;
      for (int c = 0; c < c_in; ++c)
        for (int ky = 0; ky < kh; ++ky)
          for (int kx = 0; kx < kw; ++kx) {
            const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
            row[(c * kh + ky) * kw + kx] = (iy >= 0 && iy < h && ix >= 0 && ix < w)
                                               ? in[(static_cast<size_t>(c) * h + iy) * w + ix]
                                               : 0.f;
          }
    }
  std::vector<float> out(static_cast<size_t>(c_out) * S, 0.f);
  ora_sgemm('N', 'T', c_out, static_cast<int>(S), K, 1.f, wt, K, cols.data(), K, 0.f, out.data(),
            static_cast<int>(S));
  return out;
}

// conv2d_f16 (sv.cpp:196-258): im2col rounded to fp16, gemm_f16x_fmlal.
std::vector<float> sv_conv2d_f16(const float* in, int c_in, int h, int w, const uint16_t* w16,
                                 int c_out, int kh, int kw, int stride, int pad) {
  const int oh = (h + 2 * pad - kh) / stride + 1, ow = (w + 2 * pad - kw) / stride + 1;
  const size_t S = static_cast<size_t>(oh) * ow, K = static_cast<size_t>(c_in) * kh * kw;
  std::vector<uint16_t> cols(S * K);
  for (int oy = 0; oy < oh; ++oy)
    for (int ox = 0; ox < ow; ++ox) {
      uint16_t* row = cols.data() + (static_cast<size_t>(oy) * ow + ox) * K;
      for (int c = 0; c < c_in; ++c)
        for (int ky = 0; ky < kh; ++ky)
          for (int kx = 0; kx < kw; ++kx) {
            const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
            row[(static_cast<size_t>(c) * kh + ky) * kw + kx] =
                f2h((iy >= 0 && iy < h && ix >= 0 && ix < w)
                        ? in[(static_cast<size_t>(c) * h + iy) * w + ix]
                        : 0.f);
          }
    }
  std::vector<float> out(static_cast<size_t>(c_out) * S, 0.f);
  ora_gemm_f16x_fmlal(w16, cols.data(), out.data(), static_cast<size_t>(c_out), S, K);
  return out;
}

using Named2 = std::map<std::string, const ora_named*>;

// Aff::apply (sv.cpp:445-521): att = BN2(W2 SiLU(BN1(W1 [x; ds] + b1)) + b2),
// out = x (1 + tanh att) + ds (1 - tanh att).  out may alias x.
struct SvAff {
  std::vector<uint16_t> w1, w2;
  std::vector<float> b1, b2;
  SvBn bn1, bn2;
  int inter = 0, ch = 0;
  void load(const Named2& by, const std::string& p, int c) {
    ch = c;
    w1 = sv_w16(by, p + "0.weight");
    inter = static_cast<int>(w1.size() / (2 * static_cast<size_t>(c)));
    w2 = sv_w16(by, p + "3.weight");
    b1 = sv_vec(by, p + "0.bias");
    b2 = sv_vec(by, p + "3.bias");
    bn1.load(by, p + "1");
    bn2.load(by, p + "4");
  }
  void apply(const float* x, const float* ds, float* out, size_t s) const {
    std::vector<uint16_t> xh(2 * static_cast<size_t>(ch) * s);
    for (size_t i = 0; i < s; ++i)  // f32_trans_to_f16 of cat [2ch][s] -> [s][2ch]
      for (int c = 0; c < 2 * ch; ++c)
        xh[i * 2 * ch + c] = f2h(c < ch ? x[static_cast<size_t>(c) * s + i]
                                        : ds[static_cast<size_t>(c - ch) * s + i]);
    std::vector<float> att(static_cast<size_t>(inter) * s);
    ora_gemm_f16x_fmlal(w1.data(), xh.data(), att.data(), inter, s, 2 * static_cast<size_t>(ch));
    for (int e = 0; e < inter; ++e)
      for (size_t i = 0; i < s; ++i) att[e * s + i] += b1[e];
    bn1.apply(att.data(), inter, s);
    ora_silu(att.data(), att.data(), att.size());
    std::vector<uint16_t> xh2(static_cast<size_t>(inter) * s);
    for (size_t i = 0; i < s; ++i)
      for (int e = 0; e < inter; ++e) xh2[i * inter + e] = f2h(att[static_cast<size_t>(e) * s + i]);
    std::vector<float> at(static_cast<size_t>(ch) * s);
    ora_gemm_f16x_fmlal(w2.data(), xh2.data(), at.data(), ch, s, inter);
    for (int e = 0; e < ch; ++e)
      for (size_t i = 0; i < s; ++i) at[e * s + i] += b2[e];
    bn2.apply(at.data(), ch, s);
    for (size_t i = 0; i < static_cast<size_t>(ch) * s; ++i) {
      const float t = std::tanh(at[i]);
      out[i] = x[i] * (1.0f + t) + ds[i] * (1.0f - t);
    }
  }
};

// Block::apply (sv.cpp:523-644).
struct SvBlock {
  bool aff = false, has_sc = false;
  int width = 0, scale = 4, exp = 0, stride = 1;
  std::vector<uint16_t> conv1, conv3, sc;
  std::vector<std::vector<uint16_t>> convs;
  SvBn bn1, bn3, sc_bn;
  std::vector<SvBn> bns;
  std::vector<SvAff> fuses;
  void load(const Named2& by, int l, int i, bool with_aff, int st) {
    const std::string p = "layer" + std::to_string(l) + "." + std::to_string(i) + ".";
    aff = with_aff;
    stride = st;
    bn3.load(by, p + "bn3");
    exp = static_cast<int>(bn3.g.size());
    conv1 = sv_w16(by, p + "conv1.weight");
    bn1.load(by, p + "bn1");
    width = static_cast<int>(bn1.g.size()) / scale;
    for (int j = 0; j < scale; ++j) {
      convs.push_back(sv_w16(by, p + "convs." + std::to_string(j) + ".weight"));
      bns.emplace_back();
      bns.back().load(by, p + "bns." + std::to_string(j));
    }
    conv3 = sv_w16(by, p + "conv3.weight");
    if (aff)
      for (int j = 0; j < scale - 1; ++j) {
        fuses.emplace_back();
        fuses.back().load(by, p + "fuse_models." + std::to_string(j) + ".local_att.", width);
      }
    has_sc = sv_find(by, p + "shortcut.0.weight") != nullptr;
    if (has_sc) {
      sc = sv_w16(by, p + "shortcut.0.weight");
      sc_bn.load(by, p + "shortcut.1");
    }
  }
  std::vector<float> apply(const std::vector<float>& in, int c_in, int& h, int& w) const {
    const int co1 = width * scale, h_in = h, w_in = w;
    std::vector<float> c1 = sv_conv2d_f16(in.data(), c_in, h, w, conv1.data(), co1, 1, 1, stride, 0);
    h = (h - 1) / stride + 1;
    w = (w - 1) / stride + 1;
    const size_t s = static_cast<size_t>(h) * w;
    bn1.apply(c1.data(), co1, s);
    for (float& v : c1) v = relu20f(v);
    std::vector<float> tmp2(static_cast<size_t>(co1) * s), sp(static_cast<size_t>(width) * s);
    for (int i = 0; i < scale; ++i) {
      const float* chunk = c1.data() + static_cast<size_t>(i) * width * s;
      if (i > 0) {
        if (aff)
          fuses[i - 1].apply(sp.data(), chunk, sp.data(), s);
        else
          for (size_t j = 0; j < sp.size(); ++j) sp[j] += chunk[j];
      }
      std::vector<float> nx = sv_conv2d_f16(i == 0 ? chunk : sp.data(), width, h, w,
                                            convs[i].data(), width, 3, 3, 1, 1);
      bns[i].apply(nx.data(), width, s);
      for (float& v : nx) v = relu20f(v);
      std::copy(nx.begin(), nx.end(), tmp2.begin() + static_cast<size_t>(i) * width * s);
      sp = nx;
    }
    std::vector<float> out = sv_conv2d_f16(tmp2.data(), co1, h, w, conv3.data(), exp, 1, 1, 1, 0);
    bn3.apply(out.data(), exp, s);
    if (!has_sc) {
      for (size_t j = 0; j < out.size(); ++j) out[j] += in[j];
    } else {
      std::vector<float> t = sv_conv2d_f16(in.data(), c_in, h_in, w_in, sc.data(), exp, 1, 1,
                                           stride, 0);
      sc_bn.apply(t.data(), exp, s);
      for (size_t j = 0; j < out.size(); ++j) out[j] += t[j];
    }
    for (float& v : out) v = relu20f(v);
    return out;
  }
};

size_t sv_forward(const Named2& by, const float* fbk, size_t frames, int F, float* emb_out) {
  const int T = static_cast<int>(frames);
  std::vector<float> cur(static_cast<size_t>(F) * T);
  for (int t = 0; t < T; ++t)
    for (int f = 0; f < F; ++f) cur[static_cast<size_t>(f) * T + t] = fbk[static_cast<size_t>(t) * F + f];
  const std::vector<float> w0 = sv_vec(by, "conv1.weight");
  SvBn bn1;
  bn1.load(by, "bn1");
  const int m_ch = static_cast<int>(bn1.g.size());
  std::vector<float> x = sv_conv2d_f32(cur.data(), 1, F, T, w0.data(), m_ch, 3, 3, 1, 1);
  bn1.apply(x.data(), m_ch, static_cast<size_t>(F) * T);
  for (float& v : x) v = v < 0.f ? 0.f : v;
  struct Def {
    int blocks, stride;
    bool aff;
  };
  const Def defs[4] = {{3, 1, false}, {4, 2, false}, {6, 2, true}, {3, 2, true}};
  int h = F, w = T, c = m_ch, h3 = 0, w3 = 0, c3 = 0;
  std::vector<float> o3;
  for (int l = 1; l <= 4; ++l) {
    for (int i = 0; i < defs[l - 1].blocks; ++i) {
      SvBlock b;
      b.load(by, l, i, defs[l - 1].aff, i == 0 ? defs[l - 1].stride : 1);
      x = b.apply(x, c, h, w);
      c = b.exp;
    }
    if (l == 3) {
      o3 = x;
      h3 = h, w3 = w, c3 = c;
    }
  }
  const std::vector<uint16_t> l3ds = sv_w16(by, "layer3_ds.weight");
  const std::vector<float> ds = sv_conv2d_f16(o3.data(), c3, h3, w3, l3ds.data(), c, 3, 3, 2, 1);
  SvAff f34;
  f34.load(by, "fuse34.local_att.", c);
  std::vector<float> fused(ds.size());
  f34.apply(x.data(), ds.data(), fused.data(), static_cast<size_t>(h) * w);
  for (int ci = 0; ci < c; ++ci)  // flatten (C x F) and mean over T (sv.cpp:870-879)
    for (int fy = 0; fy < h; ++fy) {
      const float* row = fused.data() + (static_cast<size_t>(ci) * h + fy) * w;
      double acc = 0.0;
      for (int t = 0; t < w; ++t) acc += row[t];
      emb_out[static_cast<size_t>(ci) * h + fy] = static_cast<float>(acc / w);
    }
  return static_cast<size_t>(c) * h;
}

}  // namespace

extern "C" size_t ora_sv_forward(const ora_named* t, size_t n, const float* fbank, size_t frames,
                                 int n_mels, float* emb) {
  Named2 by;
  for (size_t i = 0; i < n; ++i) by[t[i].name] = &t[i];
  try {
    return sv_forward(by, fbank, frames, n_mels, emb);
  } catch (const SvMissing&) {
    return 0;
  }
}

extern "C" void ora_sv_conv2d_f16(const float* in, int c_in, int h, int w, const uint16_t* w16,
                                  int c_out, int kh, int kw, int stride, int pad, float* out) {
  const std::vector<float> y = sv_conv2d_f16(in, c_in, h, w, w16, c_out, kh, kw, stride, pad);
  std::copy(y.begin(), y.end(), out);
}
