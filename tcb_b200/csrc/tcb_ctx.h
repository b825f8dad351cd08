// tcb_ctx.h - the context behind the opaque tcb_ctx handle (internal).
#pragma once

#include <stddef.h>

#include <mutex>

struct tcb_ctx {
  int dev = 0;
  int sms = 148;
  void *ws = nullptr;  // scratch owned by the context, grown on demand
  size_t ws_cap = 0;
  int *derr = nullptr;  // device error word (bounded waits that gave up)
  void *sk = nullptr;   // split-K scratch of the matvec kernels (zeroed; kernels leave it zeroed)
  size_t sk_cap = 0;
  void *hx = nullptr;   // tcb_qgemm_host: x staged on the device
  size_t hx_cap = 0;
  void *hc = nullptr;   // tcb_qgemm_host: c of a caller whose c the GPU cannot reach
  size_t hc_cap = 0;
  std::mutex mu;
  char err[256] = {0};
};
