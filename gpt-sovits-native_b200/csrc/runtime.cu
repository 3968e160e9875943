// runtime.cu — status reporting, device initialisation and the driver entry
// points (cuTensorMapEncodeTiled) the TMA paths need.
#include <cuda.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"
#include "gsvk_internal.hpp"

namespace gsvk {

namespace {
thread_local char g_err[512] = "";
thread_local int g_ready_device = -1;

struct DeviceInfo {
  int sms = 0;
  int major = 0, minor = 0;
  uint32_t* status = nullptr;  // device word written by bounded waits
};
DeviceInfo g_info[64];
std::mutex g_init_mu;
// Signature of cuTensorMapEncodeTiled (driver API, CUDA >= 12.0).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode_tiled = nullptr;
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GSVK_OK;
  return fail(GSVK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int check_launch(const char* kernel) { return check_cuda(cudaGetLastError(), kernel); }

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && g_info[dev].sms > 0) return g_info[dev].sms;
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v > 0 ? v : 148;
}

bool tma_encode_available() { return g_encode_tiled != nullptr; }

uint32_t* device_status() {
  int dev = 0;
  cudaGetDevice(&dev);
  return (dev >= 0 && dev < 64) ? g_info[dev].status : nullptr;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  if (!g_encode_tiled) return fail(GSVK_ERR_NODEV, "cuTensorMapEncodeTiled unavailable");
  uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  const CUresult r = g_encode_tiled(map, dtype, rank, base, dims, strides_bytes, box, elem_strides,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GSVK_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GSVK_OK;
}

}  // namespace gsvk

using namespace gsvk;

extern "C" {

int gsvk_version(void) { return 100; }

const char* gsvk_last_error(void) { return g_err; }

int gsvk_device_init(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return fail(GSVK_ERR_NODEV, "no CUDA device");
  }
  if (device < 0 || device >= n || device >= 64)
    return fail(GSVK_ERR_INVALID, "device %d out of range", device);
  int rc = check_cuda(cudaSetDevice(device), "cudaSetDevice");
  if (rc) return rc;
  cudaDeviceProp prop;
  rc = check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (rc) return rc;
  if (prop.major != 10)
    return fail(GSVK_ERR_NODEV, "device %d is sm_%d%d; this library is built for sm_100a", device,
                prop.major, prop.minor);
  std::lock_guard<std::mutex> lk(g_init_mu);
  g_info[device].sms = prop.multiProcessorCount;
  if (!g_info[device].status) {
    // One-time allocation at initialisation (never on the hot path).
    rc = check_cuda(cudaMalloc(&g_info[device].status, 256), "cudaMalloc(status)");
    if (rc) return rc;
    rc = check_cuda(cudaMemset(g_info[device].status, 0, 256), "cudaMemset(status)");
    if (rc) return rc;
  }
  g_info[device].major = prop.major;
  g_info[device].minor = prop.minor;
  if (!g_encode_tiled) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    rc = check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                    "cudaGetDriverEntryPoint");
    if (rc) return rc;
    if (q != cudaDriverEntryPointSuccess || !fn)
      return fail(GSVK_ERR_NODEV, "driver lacks cuTensorMapEncodeTiled");
    g_encode_tiled = reinterpret_cast<EncodeTiledFn>(fn);
  }
  g_ready_device = device;
  return GSVK_OK;
}

int gsvk_device_status(int reset) {
  uint32_t* st = device_status();
  if (!st) return fail(GSVK_ERR_NODEV, "gsvk_device_init() not called");
  uint32_t v = 0;
  int rc = check_cuda(cudaMemcpy(&v, st, 4, cudaMemcpyDeviceToHost), "read device status");
  if (rc) return rc;
  if (reset) {
    rc = check_cuda(cudaMemset(st, 0, 4), "reset device status");
    if (rc) return rc;
  }
  return v == DEV_OK ? GSVK_OK : GSVK_ERR_TIMEOUT;
}

int gsvk_available(void) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return (dev == g_ready_device || (dev >= 0 && dev < 64 && g_info[dev].sms > 0)) &&
                 g_encode_tiled != nullptr
             ? 1
             : 0;
}

}  // extern "C"
