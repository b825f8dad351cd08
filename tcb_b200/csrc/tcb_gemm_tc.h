// tcb_gemm_tc.h - the tensor-core (tcgen05) path of the float product for
// many activation rows (internal to libtcb).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

struct tcb_ctx;

namespace tcb {

// smallest M routed to the tensor-core kernel
constexpr int kTcMinM = 64;

// true when the shape, weight type and alignment suit the tcgen05 kernel
// (Q4_K dequantised in the kernel; Q6_K, Q8_0, Q4_0 dequantised exactly to
// row-scaled fp16 in workspace first)
bool tc_eligible(int wtype, int M, int N, int K, const void *w);
// the same shape and type rules for any number of rows (tc_eligible also
// asks M >= kTcMinM, the public product's routing)
bool tc_eligible_rows(int wtype, int N, int K, const void *w);
// context scratch the call needs (fp16 activations and row multipliers)
size_t tc_workspace_bytes(int wtype, int M, int N, int K);
// a step applied to the f32 activation rows as they are converted (the
// decoder's prompt pass): none, RMSNorm with weight w and eps, or SwiGLU
// over merged rows [G | U] (x rows of 2K elements, ldx >= 2K)
constexpr int kTcProNone = 0, kTcProRms = 1, kTcProSwiglu = 2;
struct TcPrologue {
  int kind = kTcProNone;
  const float *w = nullptr;
  float eps = 0.f;
};
// true when launch_qgemm_tc takes the prologue for these rows (f32, 16-byte
// aligned rows and weights, K <= 16384)
bool tc_prologue_ok(const TcPrologue &pro, int K, const void *x, long ldx);
// C (+)= X · dequant(W)^T; ws holds tc_workspace_bytes(M, N, K) bytes
cudaError_t launch_qgemm_tc(int wtype, const void *w, int M, int N, int K, const void *x, int xdt, long ldx, void *c,
                            int cdt, long ldc, int accumulate, void *ws, int *err, cudaStream_t s,
                            const TcPrologue *pro = nullptr);
// the tensor-core product of f32 rows with a prologue, through the
// context's workspace (tcb_capi.cu); TCB_ERR_UNSUPPORTED when the tensor-core
// path or the prologue does not take the shape (the caller then runs the
// step and tcb_qgemm separately)
int qgemm_tc_prologue(tcb_ctx *ctx, int wtype, int M, int N, int K, const void *w, const float *x, long ldx, float *c,
                      long ldc, int accumulate, const TcPrologue &pro, cudaStream_t s);

}  // namespace tcb
