// tcb_capi.cu - the C ABI of include/tcb.h: argument checks that TR's
// backend performs before a launch (shapes, dtypes, block alignment), the
// per-context scratch, and dispatch to the kernels.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "../../include/tcb.h"
#include "tcb_common.cuh"
#include "tcb_launch.h"
#include "tcb_ctx.h"
#include "tcb_gemm_i8.h"
#include "tcb_gemm_tc.h"
#include "tcb_matvec.h"


namespace {

int cuda_fail(tcb_ctx *ctx, cudaError_t e) {
  if (ctx) snprintf(ctx->err, sizeof ctx->err, "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return TCB_ERR_CUDA;
}

#define TCB_CU(ctx, call)                          \
  do {                                             \
    cudaError_t e_ = (call);                       \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_); \
  } while (0)

bool act_type_ok(int dt) { return dt == TCB_F32 || dt == TCB_BF16 || dt == TCB_F16; }
size_t elem_size(int dt) { return dt == TCB_F32 ? 4 : 2; }

int bind(tcb_ctx *ctx) {
  int cur = -1;
  TCB_CU(ctx, cudaGetDevice(&cur));
  if (cur != ctx->dev) TCB_CU(ctx, cudaSetDevice(ctx->dev));
  return TCB_OK;
}

// grow the context's scratch; freeing the old buffer waits for the device
int ensure_ws(tcb_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->ws_cap) return TCB_OK;
  if (ctx->ws) {
    cudaError_t e = cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_cap = 0;
    if (e != cudaSuccess) return cuda_fail(ctx, e);
  }
  size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
  cudaError_t e = cudaMalloc(&ctx->ws, cap);
  if (e != cudaSuccess) {
    cuda_fail(ctx, e);
    (void)cudaGetLastError();
    return TCB_ERR_NOMEM;
  }
  ctx->ws_cap = cap;
  return TCB_OK;
}

// grow one of the context's staging buffers (tcb_qgemm_host) to `bytes`
int ensure_buf(tcb_ctx *ctx, void **buf, size_t *cap, size_t bytes) {
  if (bytes <= *cap) return TCB_OK;
  if (*buf) {
    cudaError_t e = cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    if (e != cudaSuccess) return cuda_fail(ctx, e);
  }
  const size_t c = bytes < (64u << 10) ? (64u << 10) : bytes + (bytes >> 2);
  cudaError_t e = cudaMalloc(buf, c);
  if (e != cudaSuccess) {
    cuda_fail(ctx, e);
    (void)cudaGetLastError();
    return TCB_ERR_NOMEM;
  }
  *cap = c;
  return TCB_OK;
}

// Where memory p lives, for tcb_qgemm_host: kMemDevice (device or managed
// memory, used in place), kMemPinned (page-locked or registered host memory;
// *view is the address at which the GPU reaches it) or kMemPageable.
constexpr int kMemPageable = 0, kMemPinned = 1, kMemDevice = 2;
int mem_kind(const void *p, const void **view) {
  cudaPointerAttributes a{};
  *view = nullptr;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return kMemPageable;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    *view = p;
    return kMemDevice;
  }
  if (a.type == cudaMemoryTypeHost && a.devicePointer) {
    *view = a.devicePointer;
    return kMemPinned;
  }
  return kMemPageable;
}

// rows of x from memory the GPU reaches (pinned host memory) into a dense
// device buffer.  The previous call's product may still read dst, so the copy
// waits for the previous kernel of the stream first; the product that follows
// may launch at once (it waits for this grid before reading x).
__global__ void k_stage_rows(const uint8_t *src, long sstride, uint8_t *dst, long rowbytes, int rows) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const bool vec = (reinterpret_cast<uintptr_t>(src) | (uintptr_t)sstride | reinterpret_cast<uintptr_t>(dst) |
                    (uintptr_t)rowbytes) % 16 == 0;
  const long t0 = (long)blockIdx.x * blockDim.x + threadIdx.x, nt = (long)gridDim.x * blockDim.x;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const uint8_t *s = src + r * sstride;
    uint8_t *d = dst + r * rowbytes;
    if (vec) {
      for (long i = t0; i < rowbytes / 16; i += nt)
        reinterpret_cast<uint4 *>(d)[i] = reinterpret_cast<const uint4 *>(s)[i];
    } else {
      for (long i = t0; i < rowbytes; i += nt) d[i] = s[i];
    }
  }
}

// grow the matvec kernels' scratch to at least `bytes` (zeroed; launches
// leave it zeroed), after the device has finished with the old one
int ensure_sk(tcb_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->sk_cap) return TCB_OK;
  std::lock_guard<std::mutex> lock(ctx->mu);
  if (bytes <= ctx->sk_cap) return TCB_OK;
  if (ctx->sk) {
    TCB_CU(ctx, cudaDeviceSynchronize());
    cudaFree(ctx->sk);
    ctx->sk = nullptr;
    ctx->sk_cap = 0;
  }
  const size_t cap = bytes + (bytes >> 1);
  TCB_CU(ctx, cudaMalloc(&ctx->sk, cap));
  TCB_CU(ctx, cudaMemset(ctx->sk, 0, cap));
  ctx->sk_cap = cap;
  return TCB_OK;
}

// The TMA matvec kernels: plan, scratch, launch; *taken = false when the
// shape goes to another kernel.  They take the float product below the
// tensor-core path's minimum M and the int8-activation product at every M,
// up to 8 rows of x per launch with the weights streamed once for them.  A row's result does not depend on the other rows (the
// int8-activation fold is per row), so row groups give the same product as
// one launch over all rows.
int run_matvec(tcb_ctx *ctx, int wtype, int act8, int M, int N, int K, const void *w, const void *x, int xdt,
               long ldx, void *c, int cdt, long ldc, int accumulate, cudaStream_t s, bool *taken) {
  *taken = false;
  // the float path from kTcMinM rows on is the tensor-core product's; the
  // int8-activation product has no other fast kernel, so every M comes here
  // (the portable kernel costs about 240 us a row on the prefill shapes)
  if (M < 1 || (!act8 && M >= tcb::kTcMinM)) return TCB_OK;
  if (M > 1 && !act8 && (wtype == TCB_Q4_K || wtype == TCB_Q6_K || wtype == TCB_Q4_0) &&
      tcb::rows_plan(wtype, N, K, w, ctx->sms, 2).ok) {
    // Q4_K / Q6_K / Q4_0 float path: up to 16 rows per weight stream (fewer when
    // their digits leave too little shared memory); a last single row takes
    // the batch-1 kernel
    *taken = true;
    for (int m0 = 0, rows = 0; m0 < M; m0 += rows) {
      rows = M - m0 < 16 ? M - m0 : 16;
      tcb::MvPlan pq{};
      if (rows == 1) pq = tcb::matvec_plan(wtype, 0, 1, N, K, w, ctx->sms);
      while (!pq.ok) {
        pq = tcb::rows_plan(wtype, N, K, w, ctx->sms, rows < 2 ? 2 : rows);
        if (pq.ok) break;
        if (rows <= 2) return TCB_ERR_UNSUPPORTED;
        rows /= 2;
      }
      const void *xm = static_cast<const char *>(x) + (size_t)m0 * ldx * elem_size(xdt);
      void *cm = static_cast<char *>(c) + (size_t)m0 * ldc * elem_size(cdt);
      int rc = ensure_sk(ctx, pq.split_bytes);
      if (rc != TCB_OK) return rc;
      cudaError_t e = tcb::matvec_launch(pq, wtype, 0, N, K, w, xm, xdt, cm, cdt, accumulate, ctx->derr, s, nullptr,
                                         0, ctx->sk, rows, ldx, ldc);
      if (e != cudaSuccess) return cuda_fail(ctx, e);
    }
    return TCB_OK;
  }
  if (M > 1) {
    // the kernels take up to 8 rows per launch, streaming the weights once
    // for all of them (fewer rows per launch when their x regions leave too
    // little shared memory for the stages)
    tcb::MvPlan pq{};
    for (int mr = 8; mr >= 2 && !pq.ok; mr /= 2)
      if (mr <= 2 * M - 1 || mr == 2) pq = tcb::matvec_plan_rows(wtype, act8, N, K, w, ctx->sms, mr);
    if (pq.ok) {
      int rc = ensure_sk(ctx, pq.split_bytes);
      if (rc != TCB_OK) return rc;
      *taken = true;
      for (int m0 = 0; m0 < M; m0 += pq.rows) {
        const int rows = M - m0 < pq.rows ? M - m0 : pq.rows;
        const void *xm = static_cast<const char *>(x) + (size_t)m0 * ldx * elem_size(xdt);
        void *cm = static_cast<char *>(c) + (size_t)m0 * ldc * elem_size(cdt);
        cudaError_t e = tcb::matvec_launch(pq, wtype, act8, N, K, w, xm, xdt, cm, cdt, accumulate, ctx->derr, s,
                                           nullptr, 0, ctx->sk, rows, ldx, ldc);
        if (e != cudaSuccess) return cuda_fail(ctx, e);
      }
      return TCB_OK;
    }
  }
  tcb::MvPlan pl = tcb::matvec_plan(wtype, act8, 1, N, K, w, ctx->sms);
  if (!pl.ok) return TCB_OK;
  int rc = ensure_sk(ctx, pl.split_bytes);
  if (rc != TCB_OK) return rc;
  *taken = true;
  for (int m = 0; m < M; m++) {
    const void *xm = static_cast<const char *>(x) + (size_t)m * ldx * elem_size(xdt);
    void *cm = static_cast<char *>(c) + (size_t)m * ldc * elem_size(cdt);
    cudaError_t e =
        tcb::matvec_launch(pl, wtype, act8, N, K, w, xm, xdt, cm, cdt, accumulate, ctx->derr, s, nullptr, 0, ctx->sk);
    if (e != cudaSuccess) return cuda_fail(ctx, e);
  }
  return TCB_OK;
}

}  // namespace

namespace tcb {
// the checks TR makes before the quant product (gpu/backend_quant.go:43-65,
// tensor/quant.go:240-247, spec 15.51-15.53)
int check_gemm_args(int wtype, int M, int N, int K, const void *w, const void *x, int xdt, long ldx, void *c,
                    int cdt, long ldc) {
  int E = tcb::block_elems(wtype);
  if (!E) return TCB_ERR_DTYPE;
  if (!act_type_ok(xdt) || !act_type_ok(cdt)) return TCB_ERR_DTYPE;
  if (M < 0 || N < 0 || K < 0 || K % E) return TCB_ERR_SHAPE;
  if (M == 0 || N == 0) return TCB_OK;
  if (ldc < N || (K > 0 && ldx < K)) return TCB_ERR_SHAPE;
  if (!c || (K > 0 && (!w || !x))) return TCB_ERR_NULL;
  uintptr_t wa = reinterpret_cast<uintptr_t>(w);
  if (wa % (wtype == TCB_Q4_K ? 4 : 2)) return TCB_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(x) % elem_size(xdt) || reinterpret_cast<uintptr_t>(c) % elem_size(cdt))
    return TCB_ERR_ALIGN;
  return TCB_OK;
}

int qgemm_tc_prologue(tcb_ctx *ctx, int wtype, int M, int N, int K, const void *w, const float *x, long ldx, float *c,
                      long ldc, int accumulate, const TcPrologue &pro, cudaStream_t s) {
  if (!ctx) return TCB_ERR_NULL;
  if (M <= 0 || N <= 0 || !tc_eligible(wtype, M, N, K, w) || !tc_prologue_ok(pro, K, x, ldx) || ldc < N)
    return TCB_ERR_UNSUPPORTED;
  int rc = bind(ctx);
  if (rc != TCB_OK || (rc = ensure_ws(ctx, tc_workspace_bytes(wtype, M, N, K))) != TCB_OK) return rc;
  cudaError_t e = launch_qgemm_tc(wtype, w, M, N, K, x, TCB_F32, ldx, c, TCB_F32, ldc, accumulate, ctx->ws, ctx->derr,
                                  s, &pro);
  return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
}
}  // namespace tcb

namespace {
using tcb::check_gemm_args;

// K == 0: the empty sum; GemmSet zeroes C, Gemm leaves it
int empty_sum(tcb_ctx *ctx, int M, int N, void *c, int cdt, long ldc, int accumulate, cudaStream_t s) {
  if (accumulate || M == 0 || N == 0) return TCB_OK;
  size_t es = elem_size(cdt);
  TCB_CU(ctx, cudaMemset2DAsync(c, (size_t)ldc * es, 0, (size_t)N * es, (size_t)M, s));
  return TCB_OK;
}

}  // namespace

extern "C" {

const char *tcb_strerror(int status) {
  switch (status) {
  case TCB_OK: return "ok";
  case TCB_ERR_NULL: return "a required pointer is NULL";
  case TCB_ERR_DTYPE: return "unsupported weight, activation or output type";
  case TCB_ERR_SHAPE: return "invalid shape (negative size, K not a multiple of the block, or stride too small)";
  case TCB_ERR_ALIGN: return "pointer or offset not aligned to its element or block";
  case TCB_ERR_CUDA: return "CUDA runtime error";
  case TCB_ERR_NOMEM: return "device scratch allocation failed";
  case TCB_ERR_TIMEOUT: return "a bounded device-side wait gave up";
  case TCB_ERR_UNSUPPORTED: return "unsupported combination";
  case TCB_ERR_BOUNDS: return "index outside the table";
  case TCB_ERR_SCALE: return "NaN or Inf block scale";
  case TCB_ERR_TOO_LARGE: return "problem larger than the static scratch (TCB_STATIC_SCRATCH_BYTES)";
  }
  return "unknown status";
}

const char *tcb_last_cuda_error(tcb_ctx *ctx) { return ctx ? ctx->err : ""; }

int tcb_block_shape(int wtype, int *elems, int *bytes) {
  if (elems) *elems = tcb::block_elems(wtype);
  if (bytes) *bytes = tcb::block_bytes(wtype);
  return tcb::block_elems(wtype) ? TCB_OK : TCB_ERR_DTYPE;
}

int tcb_ctx_create(int device, tcb_ctx **out) {
  if (!out) return TCB_ERR_NULL;
  *out = nullptr;
  tcb_ctx *ctx = new (std::nothrow) tcb_ctx;
  if (!ctx) return TCB_ERR_NOMEM;
  ctx->dev = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->derr, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->derr, 0, sizeof(int));
  if (e != cudaSuccess) {
    if (ctx->derr) cudaFree(ctx->derr);
    delete ctx;
    (void)cudaGetLastError();
    return TCB_ERR_CUDA;
  }
  *out = ctx;
  return TCB_OK;
}

int tcb_device_error(tcb_ctx *ctx, int *status, int clear) {
  if (!ctx || !status) return TCB_ERR_NULL;
  *status = TCB_OK;
  if (cudaSetDevice(ctx->dev) != cudaSuccess) return TCB_ERR_CUDA;
  // every stream's work first: the word is set by kernels still in flight
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(status, ctx->derr, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(ctx->derr, 0, sizeof(int));
  if (e == cudaSuccess && clear) e = cudaDeviceSynchronize();
  return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
}

int tcb_ctx_destroy(tcb_ctx *ctx) {
  if (!ctx) return TCB_OK;
  int rc = TCB_OK;
  if (cudaSetDevice(ctx->dev) != cudaSuccess) rc = TCB_ERR_CUDA;
  for (void *p : {ctx->ws, (void *)ctx->derr, ctx->sk, ctx->hx, ctx->hc})
    if (p && cudaFree(p) != cudaSuccess) rc = TCB_ERR_CUDA;
  delete ctx;
  return rc;
}

int tcb_qgemm(tcb_ctx *ctx, int wtype, int M, int N, int K, const void *w, const void *x, int xdtype, long ldx,
              void *c, int cdtype, long ldc, int accumulate, void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  int rc = check_gemm_args(wtype, M, N, K, w, x, xdtype, ldx, c, cdtype, ldc);
  if (rc != TCB_OK || M == 0 || N == 0) return rc;
  if ((rc = bind(ctx)) != TCB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return empty_sum(ctx, M, N, c, cdtype, ldc, accumulate, s);
  bool taken = false;
  rc = run_matvec(ctx, wtype, 0, M, N, K, w, x, xdtype, ldx, c, cdtype, ldc, accumulate, s, &taken);
  if (taken || rc != TCB_OK) return rc;
  if (tcb::tc_eligible(wtype, M, N, K, w)) {
    if ((rc = ensure_ws(ctx, tcb::tc_workspace_bytes(wtype, M, N, K))) != TCB_OK) return rc;
    cudaError_t e = tcb::launch_qgemm_tc(wtype, w, M, N, K, x, xdtype, ldx, c, cdtype, ldc, accumulate, ctx->ws,
                                         ctx->derr, s);
    return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
  }
  cudaError_t e = tcb::launch_qgemm_simt(wtype, w, M, N, K, x, xdtype, ldx, c, cdtype, ldc, accumulate, ctx->sms, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e);
  return TCB_OK;
}

int tcb_qgemm_host(tcb_ctx *ctx, int wtype, int M, int N, int K, const void *w, const void *x, int xdtype, long ldx,
                   void *c, int cdtype, long ldc, int accumulate, void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  int rc = check_gemm_args(wtype, M, N, K, w, x, xdtype, ldx, c, cdtype, ldc);
  if (rc != TCB_OK || M == 0 || N == 0) return rc;
  if ((rc = bind(ctx)) != TCB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t xe = elem_size(xdtype), ce = elem_size(cdtype);
  // x: a dense device copy, made by a kernel that reads pinned memory (the
  // product then follows it without a copy-engine hand-off) or by a runtime
  // copy from pageable memory; device memory is read in place
  const void *xd = x;
  long ldxd = ldx;
  const void *view = nullptr;
  if (K > 0 && mem_kind(x, &view) != kMemDevice) {
    const long rowb = (long)K * (long)xe;
    {
      std::lock_guard<std::mutex> lock(ctx->mu);
      if ((rc = ensure_buf(ctx, &ctx->hx, &ctx->hx_cap, (size_t)M * rowb)) != TCB_OK) return rc;
    }
    if (view) {
      const long units = (rowb % 16 == 0 ? rowb / 16 : rowb);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)std::min<long>(32, std::max<long>(1, (units + 255) / 256)),
                         (unsigned)std::min(M, 65535));
      cfg.blockDim = dim3(256);
      cfg.stream = s;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      at[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      TCB_CU(ctx, cudaLaunchKernelEx(&cfg, k_stage_rows, static_cast<const uint8_t *>(view), ldx * (long)xe,
                                     static_cast<uint8_t *>(ctx->hx), rowb, M));
    } else {
      TCB_CU(ctx, cudaMemcpy2DAsync(ctx->hx, rowb, x, ldx * xe, rowb, M, cudaMemcpyHostToDevice, s));
    }
    xd = ctx->hx;
    ldxd = K;
  }
  // c: written in place where the GPU reaches it (device or pinned memory),
  // else through a device copy
  const int ck = mem_kind(c, &view);
  void *cd = ck == kMemPageable ? nullptr : const_cast<void *>(view);
  long ldcd = ldc;
  const long crow = (long)N * (long)ce;
  if (ck == kMemPageable) {
    {
      std::lock_guard<std::mutex> lock(ctx->mu);
      if ((rc = ensure_buf(ctx, &ctx->hc, &ctx->hc_cap, (size_t)M * crow)) != TCB_OK) return rc;
    }
    cd = ctx->hc;
    ldcd = N;
    if (accumulate) TCB_CU(ctx, cudaMemcpy2DAsync(cd, crow, c, ldc * ce, crow, M, cudaMemcpyHostToDevice, s));
  }
  rc = tcb_qgemm(ctx, wtype, M, N, K, w, xd, xdtype, ldxd, cd, cdtype, ldcd, accumulate, stream);
  if (rc != TCB_OK) return rc;
  if (ck == kMemPageable) TCB_CU(ctx, cudaMemcpy2DAsync(c, ldc * ce, cd, crow, crow, M, cudaMemcpyDeviceToHost, s));
  return TCB_OK;
}

int tcb_qgemm_act8(tcb_ctx *ctx, int wtype, int M, int N, int K, const void *w, const void *x, int xdtype, long ldx,
                   void *c, int cdtype, long ldc, int accumulate, void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  int rc = check_gemm_args(wtype, M, N, K, w, x, xdtype, ldx, c, cdtype, ldc);
  if (rc != TCB_OK || M == 0 || N == 0) return rc;
  if ((rc = bind(ctx)) != TCB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return empty_sum(ctx, M, N, c, cdtype, ldc, accumulate, s);
  if (tcb::i8_eligible(wtype, M, N, K, w)) {
    // many rows of Q4_K: the integer block sums on the tensor cores
    std::lock_guard<std::mutex> lock(ctx->mu);
    const size_t qb = tcb::act8_scratch_bytes(M, K, 256);
    if ((rc = ensure_ws(ctx, qb + tcb::i8_extra_bytes(M))) != TCB_OK) return rc;
    tcb::Act8Scratch sc = tcb::act8_scratch_carve(ctx->ws, M, K, 256);
    cudaError_t e = tcb::launch_act8_quantize(256, M, K, x, xdtype, ldx, sc, ctx->sms, s);
    if (e == cudaSuccess)
      e = tcb::launch_qgemm_i8(w, M, N, K, sc, static_cast<char *>(ctx->ws) + qb, x, xdtype, ldx, c, cdtype, ldc,
                               accumulate, ctx->derr, ctx->sms, s);
    return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
  }
  bool taken = false;
  rc = run_matvec(ctx, wtype, 1, M, N, K, w, x, xdtype, ldx, c, cdtype, ldc, accumulate, s, &taken);
  if (taken || rc != TCB_OK) return rc;
  const int blk = tcb::block_elems(wtype);
  std::lock_guard<std::mutex> lock(ctx->mu);
  if ((rc = ensure_ws(ctx, tcb::act8_scratch_bytes(M, K, blk))) != TCB_OK) return rc;
  tcb::Act8Scratch sc = tcb::act8_scratch_carve(ctx->ws, M, K, blk);
  cudaError_t e = tcb::launch_act8_quantize(blk, M, K, x, xdtype, ldx, sc, ctx->sms, s);
  if (e == cudaSuccess)
    e = tcb::launch_act8_dot(wtype, w, M, N, K, sc, x, xdtype, ldx, c, cdtype, ldc, accumulate, ctx->sms, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e);
  return TCB_OK;
}

int tcb_qdequant(tcb_ctx *ctx, int wtype, const void *w, long n, void *out, int odtype, void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  int E = tcb::block_elems(wtype);
  if (!E || !act_type_ok(odtype)) return TCB_ERR_DTYPE;
  if (n < 0 || n % E) return TCB_ERR_SHAPE;
  if (n == 0) return TCB_OK;
  if (!w || !out) return TCB_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(w) % 2 || reinterpret_cast<uintptr_t>(out) % elem_size(odtype)) return TCB_ERR_ALIGN;
  int rc = bind(ctx);
  if (rc != TCB_OK) return rc;
  cudaError_t e = tcb::launch_dequant_rows(wtype, w, n / E, E, nullptr, out, odtype, ctx->sms,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
}

int tcb_qembed(tcb_ctx *ctx, int wtype, const void *w, long V, int D, const int64_t *idx, int nidx, float *out,
               void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  int E = tcb::block_elems(wtype);
  if (!E) return TCB_ERR_DTYPE;
  if (V < 0 || D < 0 || nidx < 0 || D % E) return TCB_ERR_SHAPE;
  if (nidx == 0 || D == 0) return TCB_OK;
  if (!w || !idx || !out) return TCB_ERR_NULL;
  for (int i = 0; i < nidx; i++)
    if (idx[i] < 0 || idx[i] >= V) return TCB_ERR_BOUNDS;  // tensor/limits.go:30-34 (H3043)
  if (reinterpret_cast<uintptr_t>(w) % 2 || reinterpret_cast<uintptr_t>(out) % 4) return TCB_ERR_ALIGN;
  int rc = bind(ctx);
  if (rc != TCB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(ctx->mu);
  if ((rc = ensure_ws(ctx, (size_t)nidx * sizeof(int64_t))) != TCB_OK) return rc;
  int64_t *didx = static_cast<int64_t *>(ctx->ws);
  TCB_CU(ctx, cudaMemcpyAsync(didx, idx, (size_t)nidx * sizeof(int64_t), cudaMemcpyHostToDevice, s));
  cudaError_t e = tcb::launch_dequant_rows(wtype, w, nidx, D, didx, out, TCB_F32, ctx->sms, s);
  return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
}

int tcb_check_scales(int wtype, const void *host, size_t nbytes, long *bad_block) {
  if (bad_block) *bad_block = -1;
  int B = tcb::block_bytes(wtype);
  if (!B) return TCB_ERR_DTYPE;
  if (nbytes % B) return TCB_ERR_SHAPE;
  if (nbytes && !host) return TCB_ERR_NULL;
  const uint8_t *p = static_cast<const uint8_t *>(host);
  int at0 = wtype == TCB_Q6_K ? 208 : 0, at1 = wtype == TCB_Q4_K ? 2 : -1;
  for (size_t b = 0; b < nbytes / B; b++) {
    const uint8_t *blk = p + b * B;
    uint32_t s0 = blk[at0] | (blk[at0 + 1] << 8);
    bool bad = (s0 & 0x7C00u) == 0x7C00u;
    if (at1 >= 0) bad = bad || ((blk[at1] | (blk[at1 + 1] << 8)) & 0x7C00u) == 0x7C00u;
    if (bad) {
      if (bad_block) *bad_block = (long)b;
      return TCB_ERR_SCALE;
    }
  }
  return TCB_OK;
}

int tcb_quant_upload(tcb_ctx *ctx, int wtype, const void *host, size_t nbytes, void *dev, long *bad_block,
                     void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  int rc = tcb_check_scales(wtype, host, nbytes, bad_block);
  if (rc != TCB_OK || nbytes == 0) return rc;
  if (!dev) return TCB_ERR_NULL;
  if ((rc = bind(ctx)) != TCB_OK) return rc;
  TCB_CU(ctx, cudaMemcpyAsync(dev, host, nbytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
  return TCB_OK;
}

int tcb_quant_download(tcb_ctx *ctx, const void *dev, size_t nbytes, void *host, void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  if (nbytes == 0) return TCB_OK;
  if (!dev || !host) return TCB_ERR_NULL;
  int rc = bind(ctx);
  if (rc != TCB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TCB_CU(ctx, cudaMemcpyAsync(host, dev, nbytes, cudaMemcpyDeviceToHost, s));
  TCB_CU(ctx, cudaStreamSynchronize(s));
  return TCB_OK;
}

int tcb_quant_zero(tcb_ctx *ctx, int wtype, void *dev, long nblocks, void *stream) {
  if (!ctx) return TCB_ERR_NULL;
  if (!tcb::block_bytes(wtype)) return TCB_ERR_DTYPE;
  if (nblocks < 0) return TCB_ERR_SHAPE;
  if (nblocks == 0) return TCB_OK;
  if (!dev) return TCB_ERR_NULL;
  int rc = bind(ctx);
  if (rc != TCB_OK) return rc;
  cudaError_t e = tcb::launch_quant_zero(wtype, dev, nblocks, ctx->sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TCB_OK : cuda_fail(ctx, e);
}

}  // extern "C"
