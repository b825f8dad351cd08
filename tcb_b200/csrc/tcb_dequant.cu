// tcb_dequant.cu - exact dequantisation (OpenQuant), embedding rows and
// zero blocks on the device.
//
// One thread per output element: the element is rebuilt with the same
// fp32 operations, in the same order, as TR's CPU dequant
// (tensor/quant.go:139-204), including the x86 NaN rule that TR's own GPU
// kernel emulates (gpu/kernel_quant.go:13-17, 89-255).  This op is not on
// the decode hot path (it serves Open/.TR_to_dtype, embedding rows and
// tests), so it is written for exactness, not peak bandwidth.
#include "tcb_common.cuh"
#include "tcb_dequant.cuh"
#include "tcb_launch.h"

namespace tcb {

__device__ __forceinline__ void put(void *out, long i, int dt, float v) {
  if (dt == TCB_F32) static_cast<float *>(out)[i] = v;
  else if (dt == TCB_BF16) static_cast<uint16_t *>(out)[i] = f32_to_bf16(v);
  else static_cast<uint16_t *>(out)[i] = f32_to_f16(v);
}

// out[r, e] = dequant(w)[row(r), e]: rows of D elements; row(r) = r or idx[r]
template <int W>
__global__ void k_dequant_rows(const uint8_t *__restrict__ w, long rows, int D,
                               const int64_t *__restrict__ idx, void *out, int odt) {
  constexpr int E = Fmt<W>::E, B = Fmt<W>::B;
  const long rowBytes = (long)D / E * B;
  const long total = rows * (long)D;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    long r = i / D;
    int e = (int)(i - r * D);
    long src = idx ? idx[r] : r;
    const uint8_t *b = w + src * rowBytes + (long)(e / E) * B;
    put(out, i, odt, dequant_elem<W>(b, e % E));
  }
}

__global__ void k_quant_zero_q4(uint8_t *dev, long nblocks) {
  long total = nblocks * 18;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x)
    dev[i] = (i % 18) < 2 ? 0 : 0x88;
}

// any idx outside [0, V): the first offender's position, else untouched
__global__ void k_check_index(const int64_t *idx, int n, long V, int *bad) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    if (idx[i] < 0 || idx[i] >= V) atomicMin(bad, i);
}

static int grid_for(long total, int threads, int sms) {
  long g = (total + threads - 1) / threads;
  long cap = (long)sms * 16;
  return (int)(g < 1 ? 1 : g > cap ? cap : g);
}

cudaError_t launch_dequant_rows(int wtype, const void *w, long rows, int D, const int64_t *idx, void *out,
                                int odt, int sms, cudaStream_t s) {
  const int T = 256;
  int g = grid_for(rows * (long)D, T, sms);
  const uint8_t *p = static_cast<const uint8_t *>(w);
  switch (wtype) {
  case TCB_Q8_0: k_dequant_rows<TCB_Q8_0><<<g, T, 0, s>>>(p, rows, D, idx, out, odt); break;
  case TCB_Q4_0: k_dequant_rows<TCB_Q4_0><<<g, T, 0, s>>>(p, rows, D, idx, out, odt); break;
  case TCB_Q4_K: k_dequant_rows<TCB_Q4_K><<<g, T, 0, s>>>(p, rows, D, idx, out, odt); break;
  case TCB_Q6_K: k_dequant_rows<TCB_Q6_K><<<g, T, 0, s>>>(p, rows, D, idx, out, odt); break;
  default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_quant_zero(int wtype, void *dev, long nblocks, int sms, cudaStream_t s) {
  if (wtype != TCB_Q4_0) return cudaMemsetAsync(dev, 0, (size_t)nblocks * block_bytes(wtype), s);
  k_quant_zero_q4<<<grid_for(nblocks * 18, 256, sms), 256, 0, s>>>(static_cast<uint8_t *>(dev), nblocks);
  return cudaGetLastError();
}

cudaError_t launch_check_index(const int64_t *idx, int n, long V, int *bad, int sms, cudaStream_t s) {
  k_check_index<<<grid_for(n, 256, sms), 256, 0, s>>>(idx, n, V, bad);
  return cudaGetLastError();
}

}  // namespace tcb
