// C++ drop-in check: the reference's test_accel.cpp cases restated over the
// gsv::kern::cuda shim (device buffers), built against libgsvk.so.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include <cuda_runtime.h>

#include "gsv_kern_cuda.hpp"

namespace gk = gsv::kern::cuda;

static unsigned long long g_s = 0x9e3779b97f4a7c15ull;
static float rnd() {  // xorshift in [-1, 1) (test_kern.cpp:83-92 generator)
  g_s ^= g_s << 13;
  g_s ^= g_s >> 7;
  g_s ^= g_s << 17;
  return static_cast<float>(static_cast<long long>(g_s >> 40) / static_cast<double>(1ull << 23)) - 1.f;
}

template <class T>
static T* dev(const std::vector<T>& h) {
  T* d = nullptr;
  cudaMalloc(&d, h.size() * sizeof(T));
  cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
  return d;
}
template <class T>
static std::vector<T> host(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
  return h;
}

int main() {
  gk::init(0);
  int fails = 0;
  // sgemm_matches_naive_loop (test_accel.cpp:102-133)
  {
    const int M = 5, N = 7, K = 3;
    std::vector<float> A(M * K), B(K * N), C(M * N, std::nanf(""));
    for (auto& v : A) v = rnd();
    for (auto& v : B) v = rnd();
    float *dA = dev(A), *dB = dev(B), *dC = dev(C);
    gk::accel::sgemm('N', 'N', M, N, K, 1.f, dA, K, dB, N, 0.f, dC, N);
    auto got = host(dC, M * N);
    for (int i = 0; i < M; ++i)
      for (int j = 0; j < N; ++j) {
        double acc = 0;
        for (int k = 0; k < K; ++k) acc += A[i * K + k] * B[k * N + j];
        if (std::fabs(got[i * N + j] - acc) > 1e-5) ++fails;
      }
    std::vector<float> P(K * M), Q(N * K), C2(M * N, 0.5f);
    for (auto& v : P) v = rnd();
    for (auto& v : Q) v = rnd();
    float *dP = dev(P), *dQ = dev(Q), *dC2 = dev(C2);
    gk::accel::sgemm('T', 'T', M, N, K, 2.f, dP, M, dQ, K, 1.f, dC2, N);
    got = host(dC2, M * N);
    for (int i = 0; i < M; ++i)
      for (int j = 0; j < N; ++j) {
        double acc = 0;
        for (int k = 0; k < K; ++k) acc += P[k * M + i] * Q[j * K + k];
        if (std::fabs(got[i * N + j] - (2.0 * acc + 0.5)) > 1e-5) ++fails;
      }
  }
  // DenseF16 view rows == GEMV rows on fp16 activations (test_accel.cpp:135-158)
  {
    const size_t out = 128, in = 96, T = 17;
    std::vector<uint16_t> w(out * in), xh(T * in);
    for (auto& v : w) {
      const _Float16 h = static_cast<_Float16>(rnd() * 0.05f);
      std::memcpy(&v, &h, 2);
    }
    std::vector<float> x(T * in);
    for (auto& v : x) v = rnd();
    uint16_t* dw = dev(w);
    float* dx = dev(x);
    uint16_t* dxh = dev(xh);
    float* dy = dev(std::vector<float>(T * out));
    float* dyr = dev(std::vector<float>(out));
    gk::accel::DenseF16 d = gk::accel::DenseF16::view_f16(dw, out, in);
    d.forward(dx, T, dy, dxh);
    auto y = host(dy, T * out);
    for (size_t t = 0; t < T; ++t) {
      gk::gemv_f16x_fmlal(dw, dxh + t * in, dyr, out, in);
      auto yr = host(dyr, out);
      float peak = 0;
      for (float v : yr) peak = std::fmax(peak, std::fabs(v));
      for (size_t o = 0; o < out; ++o)
        if (std::fabs(y[t * out + o] - yr[o]) > 1e-5f * peak) ++fails;
    }
  }
  // pack + gemm_panel == gemm_f16x_fmlal on the same operands; batch_run runs
  // each node like its own call (gemm_f16_amx.hpp:45-78)
  {
    const size_t M = 40, N = 96, K = 128;
    std::vector<uint16_t> a(M * K), w(N * K);
    for (auto& v : a) {
      const _Float16 h = static_cast<_Float16>(rnd());
      std::memcpy(&v, &h, 2);
    }
    for (auto& v : w) {
      const _Float16 h = static_cast<_Float16>(rnd() * 0.05f);
      std::memcpy(&v, &h, 2);
    }
    uint16_t* da = dev(a);
    uint16_t* dw = dev(w);
    float* c1 = dev(std::vector<float>(M * N));
    float* c2 = dev(std::vector<float>(M * N));
    float* c3 = dev(std::vector<float>(M * N));
    gk::Panel panel = gk::pack(w.data(), N, K);  // host source: uploaded once
    gk::gemm_panel(da, panel, c1, M);
    gk::gemm_f16x_fmlal(da, dw, c2, M, N, K);
    gsvk_gemm_args node{};
    node.a = da;
    node.b = panel.data();
    node.M = M;
    node.N = N;
    node.K = K;
    node.c = c3;
    gk::batch_run(&node, 1);
    auto h1 = host(c1, M * N), h2 = host(c2, M * N), h3 = host(c3, M * N);
    for (size_t i = 0; i < M * N; ++i)
      if (h1[i] != h2[i] || h3[i] != h2[i]) ++fails;
  }
  // gemm_nt_f16w_and_dense_match_gemv_rows (test_accel.cpp:120-143): a
  // [128, 96] fp16 weight, 17 rows of fp32 activations; gemm_nt_f16w and the
  // resident DenseF16 (fp16 and fp32 constructors) against GEMV rows at
  // 1e-5 of the row peak, and bit for bit against each other.
  {
    const size_t out = 128, in = 96, T = 17;
    std::vector<uint16_t> w(out * in);
    std::vector<float> w32(out * in);
    for (size_t i = 0; i < w.size(); ++i) {
      const _Float16 h = static_cast<_Float16>(rnd() * 0.05f);
      std::memcpy(&w[i], &h, 2);
      w32[i] = static_cast<float>(h);
    }
    std::vector<float> x(T * in);
    for (auto& v : x) v = rnd();
    uint16_t* dw = dev(w);
    float* dx = dev(x);
    float* dy = dev(std::vector<float>(T * out));
    float* dyd = dev(std::vector<float>(T * out));
    float* dy32 = dev(std::vector<float>(T * out));
    float* dyv = dev(std::vector<float>(T * out));
    float* dyr = dev(std::vector<float>(out));
    gk::accel::gemm_nt_f16w(dx, T, in, dw, out, dy);
    gk::accel::DenseF16 dense(w.data(), out, in);   // host fp16 source
    dense.forward(dx, T, dyd);
    gk::accel::DenseF16 dense32(w32.data(), out, in);  // host fp32 source
    dense32.forward(dx, T, dy32);
    gk::accel::DenseF16 view = gk::accel::DenseF16::view_f16(dw, out, in);
    view.forward(dx, T, dyv);  // 3-argument view forward: f16 activations staged inside
    auto y = host(dy, T * out), yd = host(dyd, T * out), y32 = host(dy32, T * out),
         yv = host(dyv, T * out);
    uint16_t* dxh = dev(std::vector<uint16_t>(T * in));
    gk::f32_to_f16(dx, dxh, T * in);
    int f_rows = 0, f_bits = 0, f_view = 0;
    for (size_t t = 0; t < T; ++t) {
      gk::gemv_f16w_f32acc(dw, dx + t * in, dyr, out, in);
      auto yr = host(dyr, out);
      gk::gemv_f16x_fmlal(dw, dxh + t * in, dyr, out, in);
      auto yh = host(dyr, out);
      float peak = 0, peakh = 0;
      for (float v : yr) peak = std::fmax(peak, std::fabs(v));
      for (float v : yh) peakh = std::fmax(peakh, std::fabs(v));
      for (size_t o = 0; o < out; ++o) {
        const size_t i = t * out + o;
        if (std::fabs(y[i] - yr[o]) > 1e-5f * peak) ++f_rows;
        if (yd[i] != y[i] || y32[i] != y[i]) ++f_bits;            // exact widening: same bits
        if (std::fabs(yv[i] - yh[o]) > 1e-5f * peakh) ++f_view;   // view: fp16 activations
      }
    }
    gk::accel::DenseF16 moved = std::move(dense);
    moved.forward(dx, T, dyd);
    const int f_move = host(dyd, T * out) != y;
    if (f_rows || f_bits || f_view || f_move)
      std::printf("DenseF16: rows %d, bits %d, view %d, move %d\n", f_rows, f_bits, f_view, f_move);
    fails += f_rows + f_bits + f_view + f_move;
  }
  // amx_chain_run (gemm_f16_amx.hpp:90-102): two chains of three links, each
  // link reading the fp16 output of the link before it; the chain submission
  // gives the same bits as the links called one by one in order
  {
    const size_t M = 32, N = 64, K = 64;
    std::vector<uint16_t> a(M * K), w(3 * N * K);
    for (auto& v : a) {
      const _Float16 h = static_cast<_Float16>(rnd());
      std::memcpy(&v, &h, 2);
    }
    for (auto& v : w) {
      const _Float16 h = static_cast<_Float16>(rnd() * 0.1f);
      std::memcpy(&v, &h, 2);
    }
    uint16_t* da = dev(a);
    uint16_t* dw = dev(w);
    std::vector<uint16_t*> act(12);
    for (auto& p : act) p = dev(std::vector<uint16_t>(M * N));
    std::vector<float*> out(12);
    for (auto& p : out) p = dev(std::vector<float>(M * N));
    auto link = [&](int chain, int depth, int set) {
      gk::ChainLink k;
      k.chain_id = chain;
      k.depth = depth;
      k.gemm.a = depth == 0 ? da : act[set * 6 + chain * 3 + depth - 1];
      k.gemm.b = dw + static_cast<size_t>(depth) * N * K;
      k.gemm.M = M;
      k.gemm.N = N;
      k.gemm.K = K;
      k.gemm.c = out[set * 6 + chain * 3 + depth];
      k.gemm.c_f16 = act[set * 6 + chain * 3 + depth];
      k.gemm.act = chain == 0 ? GSVK_ACT_RELU : GSVK_ACT_NONE;
      return k;
    };
    std::vector<gk::ChainLink> links;
    for (int d = 2; d >= 0; --d)  // any order in the list
      for (int c = 0; c < 2; ++c) links.push_back(link(c, d, 0));
    gk::chain_run(links.data(), links.size());
    for (int c = 0; c < 2; ++c)
      for (int d = 0; d < 3; ++d) {
        const gk::ChainLink k = link(c, d, 1);
        if (gsvk_gemm_f16_ex(&k.gemm, gk::current_stream()) != GSVK_OK) ++fails;
      }
    int f_chain = 0;
    for (int i = 0; i < 6; ++i)
      if (host(out[i], M * N) != host(out[6 + i], M * N)) ++f_chain;
    if (f_chain) std::printf("chain: %d links differ\n", f_chain);
    fails += f_chain;
    // a repeated (chain, depth) pair is refused before anything runs
    std::vector<gk::ChainLink> bad = {link(0, 0, 0), link(0, 0, 0)};
    try {
      gk::chain_run(bad.data(), bad.size());
      ++fails;
    } catch (const std::runtime_error&) {
    }
  }
  // error path: a bad transpose flag throws
  try {
    gk::accel::sgemm('X', 'N', 1, 1, 1, 1.f, nullptr, 1, nullptr, 1, 0.f, nullptr, 1);
    ++fails;
  } catch (const std::runtime_error&) {
  }
  cudaDeviceSynchronize();
  std::printf("shim_test: %s (%d failures)\n", fails ? "FAIL" : "PASS", fails);
  return fails ? 1 : 0;
}
