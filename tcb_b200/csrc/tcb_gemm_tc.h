// tcb_gemm_tc.h - the tensor-core (tcgen05) path of the float product for
// many activation rows (internal to libtcb).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace tcb {

// smallest M routed to the tensor-core kernel
constexpr int kTcMinM = 64;

// true when the shape, weight type and alignment suit the tcgen05 kernel
// (Q4_K dequantised in the kernel; Q6_K, Q8_0, Q4_0 dequantised exactly to
// row-scaled fp16 in workspace first)
bool tc_eligible(int wtype, int M, int N, int K, const void *w);
// context scratch the call needs (fp16 activations and row multipliers)
size_t tc_workspace_bytes(int wtype, int M, int N, int K);
// C (+)= X · dequant(W)^T; ws holds tc_workspace_bytes(M, N, K) bytes
cudaError_t launch_qgemm_tc(int wtype, const void *w, int M, int N, int K, const void *x, int xdt, long ldx, void *c,
                            int cdt, long ldc, int accumulate, void *ws, int *err, cudaStream_t s);

}  // namespace tcb
