// tcb_static.cu - tcb_qgemm_act8_static: the int8-activation product with
// its scratch in a file-scope device array, for callers that must not
// allocate device memory (see include/tcb.h).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/tcb.h"
#include "tcb_common.cuh"
#include "tcb_launch.h"

namespace {

// The quantised activations (codes, block scales, 16-sums, finite flags)
// of one call.  In host code this name stands for the symbol, not a device
// address: kernels get the address looked up below.
__device__ __align__(256) unsigned char g_act8_scratch[TCB_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sms[kMaxDevices];  // SM count per device (0: not looked up yet)

// The scratch address is looked up on every call rather than cached: after a
// device reset the module is loaded again and the array may move.
int device_scratch(int dev, void **scratch, int *sms) {
  if (dev < 0 || dev >= kMaxDevices) return TCB_ERR_UNSUPPORTED;
  void *p = nullptr;
  if (cudaGetSymbolAddress(&p, g_act8_scratch) != cudaSuccess || !p) {
    (void)cudaGetLastError();
    return TCB_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_sms[dev] == 0 && cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    g_sms[dev] = 0;
    (void)cudaGetLastError();
    return TCB_ERR_CUDA;
  }
  *scratch = p;
  *sms = g_sms[dev];
  return TCB_OK;
}

}  // namespace

extern "C" int tcb_qgemm_act8_static(int wtype, int M, int N, int K, const void *w, const void *x, int xdtype,
                                     long ldx, void *c, int cdtype, long ldc, int accumulate, void *stream) {
  int rc = tcb::check_gemm_args(wtype, M, N, K, w, x, xdtype, ldx, c, cdtype, ldc);
  if (rc != TCB_OK || M == 0 || N == 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    if (accumulate) return TCB_OK;
    const size_t es = cdtype == TCB_F32 ? 4 : 2;
    return cudaMemset2DAsync(c, (size_t)ldc * es, 0, (size_t)N * es, (size_t)M, s) == cudaSuccess ? TCB_OK
                                                                                         : TCB_ERR_CUDA;
  }
  const int blk = tcb::block_elems(wtype);
  if (tcb::act8_scratch_bytes(M, K, blk) > TCB_STATIC_SCRATCH_BYTES) return TCB_ERR_TOO_LARGE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return TCB_ERR_CUDA;
  void *scratch = nullptr;
  int sms = 0;
  if ((rc = device_scratch(dev, &scratch, &sms)) != TCB_OK) return rc;
  // every scratch byte the dot kernel reads is written by the quantise
  // kernel of this call first (codes, scales, sums and flags of all blocks)
  const tcb::Act8Scratch sc = tcb::act8_scratch_carve(scratch, M, K, blk);
  cudaError_t e = tcb::launch_act8_quantize(blk, M, K, x, xdtype, ldx, sc, sms, s);
  if (e == cudaSuccess)
    e = tcb::launch_act8_dot(wtype, w, M, N, K, sc, x, xdtype, ldx, c, cdtype, ldc, accumulate, sms, s);
  return e == cudaSuccess ? TCB_OK : TCB_ERR_CUDA;
}
