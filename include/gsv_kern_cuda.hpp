// gsv_kern_cuda.hpp — the reference's gsv::kern / gsv::kern::accel entry
// points (src/kern/kern.hpp, gemv_fmlal.hpp, accel.hpp) re-exposed over
// libgsvk.so for DEVICE buffers, so an engine can switch its kernel calls to
// the B200 path by namespace (gsv::kern -> gsv::kern::cuda) the way it
// switches on kern::amx_gemm_available() today (gemm_f16_amx.hpp:32).
//
// Differences from the CPU originals, all deliberate:
//  - pointers are device pointers; work is queued on the calling thread's
//    current stream (set_stream), so calls return before the GPU finishes;
//  - errors throw std::runtime_error (the reference throws at load time and
//    returns silently on bad GEMM shapes, gemm_f16_amx.cpp:551-553);
//  - DenseF16 has only the view form (fp16 weights stay fp16 on the device;
//    the fp32 up-cast copy of accel.hpp:56 would double the HBM traffic).
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "gsvk.h"

namespace gsv::kern::cuda {

inline gsvk_stream_t& current_stream() {
  thread_local gsvk_stream_t s = nullptr;
  return s;
}
inline void set_stream(gsvk_stream_t s) { current_stream() = s; }

inline void check(int rc, const char* what) {
  if (rc != GSVK_OK) throw std::runtime_error(std::string(what) + ": " + gsvk_last_error());
}

// kern::amx_gemm_available() analogue: device initialised and sm_100.
inline bool available() { return gsvk_available() == 1; }
inline void init(int device = 0) { check(gsvk_device_init(device), "gsvk_device_init"); }

// kern.hpp:15
inline void gemv_f16w_f32acc(const uint16_t* w, const float* x, float* y, size_t out, size_t in) {
  check(gsvk_gemv_f16w_f32acc(w, x, y, out, in, current_stream()), "gemv_f16w_f32acc");
}
// gemv_fmlal.hpp:16
inline void f32_to_f16(const float* src, uint16_t* dst, size_t n) {
  check(gsvk_f32_to_f16(src, dst, n, current_stream()), "f32_to_f16");
}
// gemv_fmlal.hpp:26
inline void gemv_f16x_fmlal(const uint16_t* w, const uint16_t* xh, float* y, size_t out,
                            size_t in) {
  check(gsvk_gemv_f16x_fmlal(w, xh, y, out, in, current_stream()), "gemv_f16x_fmlal");
}
// gemv_fmlal.hpp:36  C[M,N] = A[M,K] . B[N,K]^T
inline void gemm_f16x_fmlal(const uint16_t* a, const uint16_t* b, float* c, size_t M, size_t N,
                            size_t K) {
  check(gsvk_gemm_f16(a, b, c, M, N, K, current_stream()), "gemm_f16x_fmlal");
}
// kern.hpp:25 (one row)
inline void layernorm(const float* x, const float* g, const float* b, float* y, size_t n,
                      double eps) {
  check(gsvk_layernorm_rows(x, g, b, y, 1, n, eps, current_stream()), "layernorm");
}
// kern.hpp:29-30
inline void softmax(const float* x, float* y, size_t n) {
  check(gsvk_softmax_rows(x, y, 1, n, current_stream()), "softmax");
}
inline void softmax_rows(const float* x, float* y, size_t rows, size_t n) {
  check(gsvk_softmax_rows(x, y, rows, n, current_stream()), "softmax_rows");
}
// kern.hpp:34
inline void relu(const float* x, float* y, size_t n) {
  check(gsvk_activation(x, y, n, GSVK_ACT_RELU, 0.f, current_stream()), "relu");
}

// AmxPanel / amx_pack (gemm_f16_amx.hpp:36-50): a weight uploaded once at
// load time; the panel owns the device copy.  Move-only, like the CPU panel.
class Panel {
 public:
  Panel() = default;
  Panel(const uint16_t* w, size_t rows, size_t cols) {
    check(gsvk_weights_register(w, rows, cols, &h_), "gsvk_weights_register");
    rows_ = rows;
    cols_ = cols;
  }
  Panel(const Panel&) = delete;
  Panel& operator=(const Panel&) = delete;
  Panel(Panel&& o) noexcept : h_(o.h_), rows_(o.rows_), cols_(o.cols_) { o.h_ = nullptr; }
  Panel& operator=(Panel&& o) noexcept {
    if (this != &o) {
      gsvk_weights_release(h_);
      h_ = o.h_;
      rows_ = o.rows_;
      cols_ = o.cols_;
      o.h_ = nullptr;
    }
    return *this;
  }
  ~Panel() { gsvk_weights_release(h_); }
  size_t rows() const { return rows_; }
  size_t cols() const { return cols_; }
  const uint16_t* data() const { return gsvk_weights_data(h_); }
  gsvk_weights_t handle() const { return h_; }

 private:
  gsvk_weights_t h_ = nullptr;
  size_t rows_ = 0, cols_ = 0;
};
// amx_pack (gemm_f16_amx.hpp:45): weights [rows, K] -> panel.
inline Panel pack(const uint16_t* w, size_t rows, size_t K) { return Panel(w, rows, K); }
// gemm_f16_amx_pp (gemm_f16_amx.hpp:56) with the weight panel as B: C = A . W^T.
inline void gemm_panel(const uint16_t* a, const Panel& w, float* c, size_t M) {
  gsvk_gemm_args g{};
  g.a = a;
  g.lda = w.cols();
  g.M = M;
  g.N = w.rows();
  g.K = w.cols();
  g.c = c;
  g.ldc = w.rows();
  g.alpha = 1.f;
  check(gsvk_gemm_f16_w(&g, w.handle(), current_stream()), "gemm_panel");
}
// amx_batch_run (gemm_f16_amx.hpp:64-78): independent GEMMs, submitted together.
inline void batch_run(const gsvk_gemm_args* nodes, size_t n) {
  check(gsvk_gemm_grouped_f16(nodes, n, current_stream()), "batch_run");
}

namespace accel {

// accel.hpp:27
inline void sgemm(char transa, char transb, int M, int N, int K, float alpha, const float* A,
                  int lda, const float* B, int ldb, float beta, float* C, int ldc) {
  check(gsvk_sgemm(transa, transb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, current_stream()),
        "sgemm");
}
// accel.hpp:33
inline void f16_to_f32(const uint16_t* src, float* dst, size_t n) {
  check(gsvk_f16_to_f32(src, dst, n, current_stream()), "f16_to_f32");
}

// accel.hpp:47-98, view form: y[T,out] = f16(x)[T,in] . W[out,in]^T with the
// fp16 activations staged in the caller's device buffer xh (>= T*in halves),
// the role the reference's std::vector<uint16_t>& xh plays.
class DenseF16 {
 public:
  DenseF16() = default;
  static DenseF16 view_f16(const uint16_t* w16_dev, size_t out, size_t in) {
    DenseF16 d;
    d.w16_ = w16_dev;
    d.out_ = out;
    d.in_ = in;
    return d;
  }
  bool is_view() const { return w16_ != nullptr; }
  const uint16_t* data_f16() const { return w16_; }
  size_t rows() const { return out_; }
  size_t cols() const { return in_; }
  void forward(const float* x, size_t T, float* y, uint16_t* xh) const {
    check(gsvk_f32_to_f16(x, xh, T * in_, current_stream()), "DenseF16 f32_to_f16");
    check(gsvk_gemm_f16(xh, w16_, y, T, out_, in_, current_stream()), "DenseF16 gemm");
  }

 private:
  const uint16_t* w16_ = nullptr;
  size_t out_ = 0, in_ = 0;
};

}  // namespace accel
}  // namespace gsv::kern::cuda
