// cwg_static.cu -- the host-buffer layer call for callers that cannot allocate
// device memory.
//
// cwg_conv3x3_fused_host needs a device workspace from the caller (the device
// copies of x and y).  Some callers cannot call cudaMalloc: code that runs
// where a framework's caching allocator owns the device heap and forbids
// outside allocations, plug-in hosts that only hand over host buffers and a
// stream, or real-time paths that may not allocate after start-up.  This file
// gives them one entry point whose staging buffer is a fixed, file-scope
// __device__ array instead, so the call itself allocates nothing.
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/cwg.h"
#include "cwg_internal.h"

namespace {

// The shared staging area: x at offset 0, y after it (256-byte aligned).
// Every GPU that loads this library holds it until the process exits.
__device__ __align__(256) unsigned char g_static_ws[CWG_STATIC_WORKSPACE_BYTES];

constexpr int kMaxDevices = 64;
void *g_ws_addr[kMaxDevices];  // device address of g_static_ws, per device
std::mutex g_ws_mu;

// The host-side name g_static_ws is only a stand-in: the device address must
// come from cudaGetSymbolAddress, once per device, with that device current.
// The address is cached for the life of the process: a device reset
// (cudaDeviceReset) after the first call is not supported, since the module
// and its array would be loaded again elsewhere.
int static_workspace(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return e == cudaErrorNoDevice ? CWG_ENODEV : CWG_ECUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return CWG_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_ws_mu);
  if (!g_ws_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_ws);
    if (e != cudaSuccess || !p) {
      cwgk_set_cuda_error((int)e);
      return CWG_ECUDA;
    }
    g_ws_addr[dev] = p;
  }
  *out = g_ws_addr[dev];
  return CWG_OK;
}

}  // namespace

extern "C" int cwg_conv3x3_fused_host_static(const void *x_host, const void *U,
                                             const float *bias, void *y_host, int n, int c_in,
                                             int c_out, int h, int w, int m, unsigned flags,
                                             void *stream) {
  if (n == 0 && c_in > 0 && c_out > 0 && h > 0 && w > 0) return CWG_OK;  // empty batch
  const size_t need = cwg_host_workspace_bytes(n, c_in, c_out, h, w, flags);
  if (need == 0 || !x_host || !y_host) return CWG_EINVAL;
  if (need > (size_t)CWG_STATIC_WORKSPACE_BYTES) return CWG_EUNSUPPORTED;
  void *ws = nullptr;
  const int rc = static_workspace(&ws);
  if (rc != CWG_OK) return rc;
  // The array used is the current device's: a stream of another device could
  // not reach it.
  if (stream) {
    int sdev = -1, dev = -1;
    cudaError_t e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev);
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
      cwgk_set_cuda_error((int)e);
      return CWG_ECUDA;
    }
    if (sdev != dev) return CWG_EINVAL;
  }
  // x and y are overwritten in full by the copy-in and by the kernel, so the
  // previous call's contents never leak into this one.  One stream, nothing
  // created or allocated.
  const size_t esz = (flags & CWG_BF16) ? 2 : 4;
  const size_t xbytes = (size_t)n * c_in * h * w * esz;
  const size_t ybytes = (size_t)n * c_out * h * w * esz;
  char *xd = static_cast<char *>(ws);
  char *yd = xd + (xbytes + 255) / 256 * 256;
  return cwgh_conv_host_serial(x_host, U, bias, y_host, xd, yd, xbytes, ybytes, n, c_in, c_out,
                               h, w, m, flags, stream);
}
