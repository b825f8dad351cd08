// tcb_matvec.h - the tensor-core matvec path (batch 1) of libtcb.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace tcb {

// launch plan of the batch-1 tensor-core kernel; ok == false when the
// shape is not taken by it (the caller then runs the portable kernel)
struct MvPlan {
  bool ok;
  int kind;                    // 0: generic kernel, 1: Q4_K float kernel, 2: Q6_K float kernel,
                               // 3: Q4_K float kernel of 2..16 rows (tcb_mv_rows.cu)
  int tiles, cbc, nch;         // tiles, blocks per staged chunk, chunks per row
  int stages, pitch;           // TMA stages, bytes per staged row
  int xoff, toff, soff, smem;  // shared-memory layout
  int grid;
  int ksplit, cpk;             // K splits and chunks per split (kind 2); 1 when not split
  size_t split_bytes;          // device scratch a launch needs (zeroed once; launches leave it zeroed), 0 if none
  int rows, xstride;           // kind 1: rows of x a launch takes, bytes between their digit regions
  int pair;                    // kind 1: F when the launch pairs gate and up rows for SwiGLU, else 0
  long ldw;                    // kind 0: bytes from one weight row to the next (the packed row size,
                               // or a padded pitch given to the planner)
  alignas(64) unsigned char tmap[128];  // TMA descriptor of the weight (CUtensorMap)
};

// smallest N that takes the Q6_K float kernel (kind 2)
constexpr int kQ6kMinRows = 32768;

// The matvec kernels' scratch (plan.split_bytes, shared by every launch of a
// context or decoder): [0, kScratchCntBytes) arrival counters, which start at
// zero and are left at zero by every launch, then partial sums, which any
// launch may overwrite.  The layout does not depend on the shape, so one
// launch's partials never land on another's counters.
constexpr size_t kScratchCntBytes = 1024;

// ldw: bytes between weight rows when they are not packed (0: packed).  A
// 2-D TMA map needs a row stride that is a multiple of 16 bytes, which a
// Q6_K row (210 bytes a block) is only for a multiple of 8 blocks; a copy
// with each row padded to a multiple of 16 bytes is read through the generic
// kernel with ldw = its pitch (Q6_K float path only; other cases refuse).
MvPlan matvec_plan(int wtype, int act8, int M, int N, int K, const void *w, int sms, long ldw = 0);
// up to mr (2, 4, 8) rows of x per launch streaming the weights once, float
// or int8-activation path (ok = false when the rows' x regions leave too
// little shared memory, or for the wide Q6_K kernel)
MvPlan matvec_plan_rows(int wtype, int act8, int N, int K, const void *w, int sms, int mr, long ldw = 0);

// Q4_K float path (kind 1).  With nw, the product is W * rms(x): an
// RMSNorm (x / sqrt(mean(x^2) + eps) * nw, K elements, f32 x, finite x
// assumed) is fused into the prologue.
// mr (1, 2, 4, 8): the most rows of x one launch takes; a launch of M <= mr
// rows (row strides ldx, ldc) streams the weights once for all of them.
// scratch: plan.split_bytes of the matvec scratch (none for this kernel).
// pair = F: the weight holds gate rows then up rows, F each (N = 2F, F a
// multiple of 16), and the launch (M = 1, f32 x, no accumulate) writes
// swi[i] = silu(g_i) * u_i for i < F instead of c: a tile stages gate rows
// 16t.. and up rows F + 16t.. side by side (two 16-row boxes).
MvPlan q4k_plan(int N, int K, const void *w, int sms, int mr = 1, int pair = 0);
cudaError_t q4k_launch(const MvPlan &pl, int N, int K, const void *w, const void *x, int xdt, void *c, int cdt,
                       int accumulate, int *err, void *scratch, cudaStream_t s, const float *nw = nullptr,
                       float eps = 0.f, const void *pf = nullptr, size_t pf_bytes = 0, int M = 1, long ldx = 0,
                       long ldc = 0, float *swi = nullptr);

// Q6_K float path (kind 2; taken from kQ6kMinRows rows, the output head;
// the plan refuses products of fewer tiles than half the SMs).
MvPlan q6k_plan(int N, int K, const void *w, int sms);
cudaError_t q6k_launch(const MvPlan &pl, int N, int K, const void *w, const void *x, int xdt, void *c, int cdt,
                       int accumulate, int *err, cudaStream_t s, const void *pf = nullptr, size_t pf_bytes = 0,
                       void *scratch = nullptr);

// Q4_K / Q6_K / Q4_0 float path of 2..16 rows of x in one weight stream (kind 3): the
// digitising prologue, the product and (when plan.ksplit > 1) the sum of the
// K-range partials, three launches on s.  plan.rows (4, 8, 12, 16) is the
// most rows a launch takes; the launch needs plan.split_bytes of scratch
// (its counter region untouched).
MvPlan rows_plan(int wtype, int N, int K, const void *w, int sms, int M);
cudaError_t rows_launch(const MvPlan &pl, int N, int K, const void *w, const void *x, int xdt, long ldx, void *c,
                        int cdt, long ldc, int accumulate, int M, int *err, void *scratch, cudaStream_t s);

// pf / pf_bytes: the weights of the next kernel of a chain, streamed into L2
// by this launch's producers (a hint; nullptr for none)
cudaError_t matvec_launch(const MvPlan &pl, int wtype, int act8, int N, int K, const void *w, const void *x, int xdt,
                          void *c, int cdt, int accumulate, int *err, cudaStream_t s, const void *pf = nullptr,
                          size_t pf_bytes = 0, void *scratch = nullptr, int M = 1, long ldx = 0, long ldc = 0);

}  // namespace tcb
