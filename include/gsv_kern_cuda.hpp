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
//  - the resident DenseF16 built from fp16 weights (accel.hpp:53) keeps them
//    fp16 on the device and widens them exactly inside the GEMM
//    (gemm_nt_f16w), which gives the sgemm results of the reference's fp32
//    up-cast copy without storing (and streaming) twice the bytes;
//  - AmxChainLink's host-side `prepare` hook has no counterpart (operands are
//    device tensors written by the previous link's epilogue).
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

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
// AmxChainLink / amx_chain_run (gemm_f16_amx.hpp:90-102): links of one chain
// run in depth order, chains are independent.
struct ChainLink {
  int chain_id = 0;
  int depth = 0;
  gsvk_gemm_args gemm{};
};
inline void chain_run(const ChainLink* links, size_t n) {
  static_assert(sizeof(ChainLink) == sizeof(gsvk_gemm_chain_link), "ChainLink layout");
  check(gsvk_gemm_chain_run(reinterpret_cast<const gsvk_gemm_chain_link*>(links), n,
                            current_stream()),
        "chain_run");
}
// AmxTileChainLink / amx_tile_chain_run (gemm_f16_amx.hpp:104-124): the
// reference's per-tile prepare overlap is the TMA / MMA pipeline inside each
// link's kernel, so the same submission serves both.
using TileChainLink = ChainLink;
inline void tile_chain_run(const TileChainLink* links, size_t n) { chain_run(links, n); }

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

// accel.hpp:38-41  y[T,out] = x[T,in] . W[out,in]^T, W fp16 widened exactly.
inline void gemm_nt_f16w(const float* x, size_t T, size_t in, const uint16_t* w, size_t out,
                         float* y) {
  check(gsvk_gemm_nt_f16w(x, T, in, w, out, y, current_stream()), "gemm_nt_f16w");
}

// accel.hpp:47-98.  Three forms, as in the reference:
//  - view (view_f16): borrows fp16 weights; forward = f16(x) . W^T on the
//    tensor cores, the fp16 activations staged in the caller's device buffer
//    xh (>= T*in halves, the role of the reference's std::vector xh);
//  - resident from fp16 weights (accel.hpp:53): owns a device copy of the
//    fp16 weights; forward = gemm_nt_f16w (fp32 activations);
//  - resident from fp32 weights (accel.hpp:54): owns a device fp32 copy;
//    forward = sgemm.
// Source pointers of the owning constructors may be host or device memory.
// The 3-argument forward of a view stages its fp16 activations in a device
// buffer the object grows on first use (the reference allocates a vector on
// every such call).  Move-only.
class DenseF16 {
 public:
  DenseF16() = default;
  DenseF16(const uint16_t* w16, size_t out, size_t in) : out_(out), in_(in) {
    check(gsvk_weights_register(w16, out, in, &panel_), "DenseF16(w16)");
  }
  DenseF16(const float* w32_src, size_t out, size_t in) : out_(out), in_(in) {
    void* p = nullptr;
    check(gsvk_device_alloc_copy(w32_src, out * in * sizeof(float), &p), "DenseF16(w32)");
    w32_ = static_cast<float*>(p);
  }
  static DenseF16 view_f16(const uint16_t* w16_dev, size_t out, size_t in) {
    DenseF16 d;
    d.w16_ = w16_dev;
    d.out_ = out;
    d.in_ = in;
    return d;
  }
  DenseF16(const DenseF16&) = delete;
  DenseF16& operator=(const DenseF16&) = delete;
  DenseF16(DenseF16&& o) noexcept { *this = std::move(o); }
  DenseF16& operator=(DenseF16&& o) noexcept {
    if (this != &o) {
      release();
      w16_ = o.w16_;
      panel_ = o.panel_;
      w32_ = o.w32_;
      xh_ = o.xh_;
      xh_cap_ = o.xh_cap_;
      out_ = o.out_;
      in_ = o.in_;
      o.w16_ = nullptr;
      o.panel_ = nullptr;
      o.w32_ = nullptr;
      o.xh_ = nullptr;
      o.xh_cap_ = 0;
    }
    return *this;
  }
  ~DenseF16() { release(); }

  bool is_view() const { return w16_ != nullptr; }
  const uint16_t* data_f16() const { return w16_ ? w16_ : (panel_ ? gsvk_weights_data(panel_) : nullptr); }
  size_t rows() const { return out_; }
  size_t cols() const { return in_; }

  // y[T,out] = x[T,in] . W^T; y is overwritten.
  void forward(const float* x, size_t T, float* y, uint16_t* xh) const {
    if (!w16_) {
      forward(x, T, y);
      return;
    }
    check(gsvk_f32_to_f16(x, xh, T * in_, current_stream()), "DenseF16 f32_to_f16");
    check(gsvk_gemm_f16(xh, w16_, y, T, out_, in_, current_stream()), "DenseF16 gemm");
  }
  void forward(const float* x, size_t T, float* y) {
    if (w16_) {
      if (xh_cap_ < T * in_) {
        gsvk_device_free(xh_);
        xh_ = nullptr;
        xh_cap_ = 0;
        void* p = nullptr;
        check(gsvk_device_alloc_copy(nullptr, T * in_ * 2, &p), "DenseF16 activation buffer");
        xh_ = static_cast<uint16_t*>(p);
        xh_cap_ = T * in_;
      }
      forward(x, T, y, xh_);
      return;
    }
    if (panel_) {
      gemm_nt_f16w(x, T, in_, gsvk_weights_data(panel_), out_, y);
      return;
    }
    if (!w32_) throw std::runtime_error("DenseF16::forward on an empty object");
    sgemm('N', 'T', static_cast<int>(T), static_cast<int>(out_), static_cast<int>(in_), 1.0f, x,
          static_cast<int>(in_), w32_, static_cast<int>(in_), 0.0f, y, static_cast<int>(out_));
  }
  void forward(const float* x, size_t T, float* y) const {
    if (w16_) throw std::runtime_error("DenseF16::forward (const view) needs an xh buffer");
    const_cast<DenseF16*>(this)->forward(x, T, y);
  }

 private:
  void release() {
    if (panel_) gsvk_weights_release(panel_);
    if (w32_) gsvk_device_free(w32_);
    if (xh_) gsvk_device_free(xh_);
    panel_ = nullptr;
    w32_ = nullptr;
    xh_ = nullptr;
    xh_cap_ = 0;
  }
  const uint16_t* w16_ = nullptr;  // view
  gsvk_weights_t panel_ = nullptr; // resident fp16
  float* w32_ = nullptr;           // resident fp32
  uint16_t* xh_ = nullptr;         // view: staged activations of the 3-argument forward
  size_t xh_cap_ = 0;
  size_t out_ = 0, in_ = 0;
};

}  // namespace accel
}  // namespace gsv::kern::cuda
