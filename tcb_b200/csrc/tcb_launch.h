// tcb_launch.h - host-side launchers of the quantized-path kernels
// (internal to libtcb; the public boundary is include/tcb.h).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tcb {

// scratch for the int8-activation path of M rows of K elements, blk the
// activation block (32 or 256)
struct Act8Scratch {
  int8_t *q8;      // [M][K] codes
  float *d8;       // [M][K/blk] block scales
  int16_t *bs;     // [M][K/16] sums of 16 codes
  uint8_t *flags;  // [M][K/blk] 1 = block finite
};
size_t act8_scratch_bytes(int M, int K, int blk);
// argument checks shared by the products' entry points (TCB_OK or an error)
int check_gemm_args(int wtype, int M, int N, int K, const void *w, const void *x, int xdt, long ldx, void *c,
                    int cdt, long ldc);
Act8Scratch act8_scratch_carve(void *base, int M, int K, int blk);

cudaError_t launch_dequant_rows(int wtype, const void *w, long rows, int D, const int64_t *idx, void *out,
                                int odt, int sms, cudaStream_t s);
cudaError_t launch_quant_zero(int wtype, void *dev, long nblocks, int sms, cudaStream_t s);
cudaError_t launch_check_index(const int64_t *idx, int n, long V, int *bad, int sms, cudaStream_t s);

// float path, portable kernel (any 2/4-byte aligned rows)
cudaError_t launch_qgemm_simt(int wtype, const void *w, int M, int N, int K, const void *x, int xdt, long ldx,
                              void *c, int cdt, long ldc, int accumulate, int sms, cudaStream_t s);

// int8-activation path
cudaError_t launch_act8_quantize(int blk, int M, int K, const void *x, int xdt, long ldx, const Act8Scratch &sc,
                                 int sms, cudaStream_t s);
cudaError_t launch_act8_dot(int wtype, const void *w, int M, int N, int K, const Act8Scratch &sc, const void *x,
                            int xdt, long ldx, void *c, int cdt, long ldc, int accumulate, int sms,
                            cudaStream_t s);

// causal grouped-query attention of M prompt rows (positions p0 ..) over one
// layer's fp16 cache [KVH][max_ctx][128] (tcb_attn_prefill.cu)
cudaError_t launch_attn_prefill(const float *q, long ldq, const __half *kc, const __half *vc, float *out, long ldo,
                                int p0, int M, int H, int KVH, int max_ctx, cudaStream_t s);

}  // namespace tcb
