// registry.cu — weight registration (the analogue of amx_pack / AmxPanel,
// gemm_f16_amx.hpp:36-50: a one-off upload at load time that the GEMM / GEMV
// calls then borrow) and the grouped GEMM (amx_batch_run,
// gemm_f16_amx.hpp:64-78: independent GEMMs submitted together).
//
// A registered matrix is a device copy of a row-major [rows, cols] fp16
// weight — the layout the TMA descriptors read directly, so no re-packing is
// needed (the conv weights' tap-major packing has its own entry points).
#include <cstring>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_weights {
  uint16_t* dev = nullptr;
  size_t rows = 0, cols = 0;
};

using namespace gsvk;

extern "C" {

int gsvk_weights_register(const uint16_t* w, size_t rows, size_t cols, gsvk_weights_t* out) {
  if (!w || !out || rows == 0 || cols == 0)
    return fail(GSVK_ERR_INVALID, "weights_register: null pointer or empty matrix");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  auto* h = new gsvk_weights();
  h->rows = rows;
  h->cols = cols;
  const size_t bytes = rows * cols * 2;
  if (cudaMalloc(&h->dev, bytes) != cudaSuccess) {
    cudaGetLastError();
    delete h;
    return fail(GSVK_ERR_NOMEM, "weights_register: %zu bytes", bytes);
  }
  // host or device source (unified addressing); synchronous, like the
  // reference's load-time packing
  if (int rc = check_cuda(cudaMemcpy(h->dev, w, bytes, cudaMemcpyDefault), "weights upload")) {
    cudaFree(h->dev);
    delete h;
    return rc;
  }
  *out = h;
  return GSVK_OK;
}

int gsvk_weights_release(gsvk_weights_t h) {
  if (!h) return GSVK_OK;
  if (h->dev) cudaFree(h->dev);
  delete h;
  return GSVK_OK;
}

const uint16_t* gsvk_weights_data(gsvk_weights_t h) { return h ? h->dev : nullptr; }

int gsvk_gemm_f16_w(const gsvk_gemm_args* args, gsvk_weights_t w, gsvk_stream_t stream) {
  if (!args || !w) return fail(GSVK_ERR_INVALID, "gemm_f16_w: null argument");
  if (args->N != w->rows || args->K != w->cols)
    return fail(GSVK_ERR_INVALID, "gemm_f16_w: N x K = %zu x %zu but the weights are %zu x %zu",
                args->N, args->K, w->rows, w->cols);
  gsvk_gemm_args g = *args;
  g.b = w->dev;
  g.ldb = w->cols;
  return gemm_ex_run(&g, as_cuda(stream), true);  // registered weights are immutable
}

int gsvk_gemv_f16w_f32acc_w(gsvk_weights_t w, const float* x, float* y, gsvk_stream_t stream) {
  if (!w) return fail(GSVK_ERR_INVALID, "gemv_f16w_f32acc_w: null weights");
  return gsvk_gemv_f16w_f32acc(w->dev, x, y, w->rows, w->cols, stream);
}

int gsvk_device_alloc_copy(const void* src, size_t bytes, void** out) {
  if (!out || bytes == 0) return fail(GSVK_ERR_INVALID, "device_alloc_copy: null out or empty");
  *out = nullptr;
  if (!gsvk_available()) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(GSVK_ERR_NOMEM, "device_alloc_copy: %zu bytes", bytes);
  }
  const int rc = src ? check_cuda(cudaMemcpy(p, src, bytes, cudaMemcpyDefault), "device upload")
                     : check_cuda(cudaMemset(p, 0, bytes), "device memset");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *out = p;
  return GSVK_OK;
}

int gsvk_device_free(void* p) {
  if (!p) return GSVK_OK;
  return check_cuda(cudaFree(p), "device_free");
}

int gsvk_gemm_chain_run(const gsvk_gemm_chain_link* links, size_t n, gsvk_stream_t stream) {
  if (n && !links) return fail(GSVK_ERR_INVALID, "gemm_chain_run: null link list");
  // validate everything first: a bad link launches nothing
  int max_depth = -1;
  for (size_t i = 0; i < n; ++i) {
    const gsvk_gemm_chain_link& k = links[i];
    if (k.depth < 0 || k.depth > 4095)
      return fail(GSVK_ERR_INVALID, "gemm_chain_run: link %zu has depth %d", i, k.depth);
    for (size_t j = 0; j < i; ++j)
      if (links[j].chain_id == k.chain_id && links[j].depth == k.depth)
        return fail(GSVK_ERR_INVALID, "gemm_chain_run: links %zu and %zu share chain %d depth %d",
                    j, i, k.chain_id, k.depth);
    const gsvk_gemm_args& g = k.gemm;
    if (!g.a || !g.b || (!g.c && !g.c_f16) || g.M == 0 || g.N == 0 || g.K == 0 ||
        (g.lda && g.lda < g.K) || (g.ldb && g.ldb < g.K))
      return fail(GSVK_ERR_INVALID, "gemm_chain_run: link %zu is invalid", i);
    if (k.depth > max_depth) max_depth = k.depth;
  }
  // Depth level by level on the stream: every link of depth d follows every
  // link of depth d - 1 (so each chain runs in order), and the links of one
  // level are independent problems launched back to back.
  std::vector<gsvk_gemm_args> level;
  for (int d = 0; d <= max_depth; ++d) {
    level.clear();
    for (size_t i = 0; i < n; ++i)
      if (links[i].depth == d) level.push_back(links[i].gemm);
    if (!level.empty())
      if (int rc = gsvk_gemm_grouped_f16(level.data(), level.size(), stream)) return rc;
  }
  return GSVK_OK;
}

int gsvk_gemm_grouped_f16(const gsvk_gemm_args* groups, size_t count, gsvk_stream_t stream) {
  if (count && !groups) return fail(GSVK_ERR_INVALID, "gemm_grouped_f16: null group list");
  // validate every group before launching any, so a bad group launches nothing
  for (size_t i = 0; i < count; ++i) {
    const gsvk_gemm_args& g = groups[i];
    if (!g.a || !g.b || (!g.c && !g.c_f16) || g.M == 0 || g.N == 0 || g.K == 0 ||
        (g.lda && g.lda < g.K) || (g.ldb && g.ldb < g.K))
      return fail(GSVK_ERR_INVALID, "gemm_grouped_f16: group %zu is invalid", i);
  }
  for (size_t i = 0; i < count; ++i) {
    gsvk_gemm_args g = groups[i];
    if (!g.lda) g.lda = g.K;
    if (!g.ldb) g.ldb = g.K;
    if (int rc = gsvk_gemm_f16_ex(&g, stream)) return rc;
  }
  return GSVK_OK;
}

}  // extern "C"
