// tcb_gemm_i8.h - the int8-activation product of many rows on the tensor
// cores (Q4_K weights; internal to libtcb).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "tcb_launch.h"

namespace tcb {

// rows from which tcb_qgemm_act8 takes the tensor-core kernel
constexpr int kI8MinM = 64;
// true when launch_qgemm_i8 takes the product (Q4_K, M >= kI8MinM, 16-byte
// aligned weights)
bool i8_eligible(int wtype, int M, int N, int K, const void *w);
// device scratch beyond the activation codes (act8_scratch_bytes): per-row
// finite flags and a count of the rows that are not
size_t i8_extra_bytes(int M);
// c (+)= quantGemmQ8 of the activations quantised into sc (launch_act8_quantize
// with 256-element blocks): the tensor-core kernel for the finite rows, TR's
// float path for the others.  extra: i8_extra_bytes(M) of device scratch.
cudaError_t launch_qgemm_i8(const void *w, int M, int N, int K, const Act8Scratch &sc, void *extra, const void *x,
                            int xdt, long ldx, void *c, int cdt, long ldc, int accumulate, int *err, int sms,
                            cudaStream_t s);

}  // namespace tcb
