"""tcb_b200 - B200 (sm_100a) quantized-tensor path of TR (sekerahmet/TCB).

The product is the C library ``tcb_b200/libtcb.so`` (include/tcb.h).  This
module is a thin ctypes view of that ABI for Python callers, tests and the
benchmark; it holds no arithmetic of its own and never falls back to the
CPU: if the library is missing it raises.

Names follow TR's tensor.Backend quant branch:
  qgemm       Backend.Gemm / GemmSet with quantized b (gpu/backend_quant.go:43)
  qgemm_act8  ActQuantGemmer.GemmActQuant (tensor/matmul.go:59-61)
  qdequant    QuantOpener.OpenQuant (tensor/quant.go:103-105)
  qembed      Backend.Embedding with quantized w (tensor/limits.go:15-45)
  quant_upload / quant_download   FromRaw / ToRaw (gpu/typed.go:24-55)
  quant_zero  QuantZeroRaw on the device (tensor/quant.go:416-427)
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtcb.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "tcb.h")

Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14
F32, F16, BF16 = 0, 1, 30
BLOCK = {Q8_0: (32, 34), Q4_0: (32, 18), Q4_K: (256, 144), Q6_K: (256, 210)}
NAMES = {Q8_0: "q8_0", Q4_0: "q4_0", Q4_K: "q4_k", Q6_K: "q6_k"}

STATUS = {
    0: "TCB_OK", 1: "TCB_ERR_NULL", 2: "TCB_ERR_DTYPE", 3: "TCB_ERR_SHAPE", 4: "TCB_ERR_ALIGN",
    5: "TCB_ERR_CUDA", 6: "TCB_ERR_NOMEM", 7: "TCB_ERR_TIMEOUT", 8: "TCB_ERR_UNSUPPORTED",
    9: "TCB_ERR_BOUNDS", 10: "TCB_ERR_SCALE", 11: "TCB_ERR_TOO_LARGE",
}


class TcbError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: {STATUS.get(code, code)} ({what_msg(code)})")
        self.code = code


_lib = None


def what_msg(code: int) -> str:
    return lib().tcb_strerror(code).decode()


def header_symbols() -> list[str]:
    """Every function declared in include/tcb.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|const char \*)\s*(tcb_\w+)\(", text, re.M)))


def lib() -> ctypes.CDLL:
    """Load libtcb.so from the package directory (build it with
    ``python -m tcb_b200.build``).  No fallback: a missing library raises."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; build it with `python -m tcb_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    P, I, Lg, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_size_t
    L.tcb_strerror.restype = ctypes.c_char_p
    L.tcb_strerror.argtypes = [I]
    L.tcb_last_cuda_error.restype = ctypes.c_char_p
    L.tcb_last_cuda_error.argtypes = [P]
    L.tcb_ctx_create.argtypes = [I, ctypes.POINTER(P)]
    L.tcb_ctx_destroy.argtypes = [P]
    L.tcb_device_error.argtypes = [P, ctypes.POINTER(I), I]
    L.tcb_peer_ar_selftest.argtypes = [P, I, I, I, ctypes.c_uint, P]
    L.tcb_block_shape.argtypes = [I, ctypes.POINTER(I), ctypes.POINTER(I)]
    L.tcb_qgemm.argtypes = [P, I, I, I, I, P, P, I, Lg, P, I, Lg, I, P]
    L.tcb_qgemm_act8.argtypes = [P, I, I, I, I, P, P, I, Lg, P, I, Lg, I, P]
    L.tcb_qgemm_host.argtypes = [P, I, I, I, I, P, P, I, Lg, P, I, Lg, I, P]
    L.tcb_qgemm_act8_static.argtypes = [I, I, I, I, P, P, I, Lg, P, I, Lg, I, P]
    L.tcb_qdequant.argtypes = [P, I, P, Lg, P, I, P]
    L.tcb_qembed.argtypes = [P, I, P, Lg, I, P, I, P, P]
    L.tcb_quant_upload.argtypes = [P, I, P, Z, P, ctypes.POINTER(Lg), P]
    L.tcb_quant_download.argtypes = [P, P, Z, P, P]
    L.tcb_quant_zero.argtypes = [P, I, P, Lg, P]
    L.tcb_check_scales.argtypes = [I, P, Z, ctypes.POINTER(Lg)]
    _lib = L
    return L


def _ptr(t) -> int:
    """Device/host address of a torch tensor, numpy array or int."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    raise TypeError(type(t))


def _dtype_code(t) -> int:
    import torch

    return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}[t.dtype]


def _stream(stream) -> int:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def row_bytes(wtype: int, K: int) -> int:
    e, b = BLOCK[wtype]
    return K // e * b


class Context:
    """One tcb_ctx: binds a device and owns the scratch of its calls."""

    def __init__(self, device: int = 0):
        self._h = ctypes.c_void_p()
        rc = lib().tcb_ctx_create(device, ctypes.byref(self._h))
        if rc:
            raise TcbError(rc, "tcb_ctx_create")
        self.device = device

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib().tcb_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_error(self, clear: bool = False) -> int:
        """The status a kernel of this context recorded when a bounded
        device-side wait gave up (0 = none); waits for the device first."""
        st = ctypes.c_int(0)
        self._check(lib().tcb_device_error(self._h, ctypes.byref(st), int(clear)), "tcb_device_error")
        return st.value

    def peer_ar_selftest(self, tp: int, rank: int, d_model: int, polls: int, stream=None):
        """tcb_peer_ar_selftest: one peer all-reduce with every rank's buffer
        local to this device, each wait limited to `polls` polls (tp > 1:
        the other ranks never arrive, so the waits give up)."""
        self._check(lib().tcb_peer_ar_selftest(self._h, tp, rank, d_model, polls, _stream(stream)),
                    "tcb_peer_ar_selftest")

    def _check(self, rc: int, what: str):
        if rc:
            err = TcbError(rc, what)
            if rc == 5:
                err.args = (err.args[0] + ": " + lib().tcb_last_cuda_error(self._h).decode(),)
            raise err

    # -- products ----------------------------------------------------------
    def qgemm(self, wtype, w, x, c, N=None, K=None, accumulate=False, stream=None, act8=False):
        """c[M,N] (+)= x[M,K] . dequant(w)^T ; x, c torch CUDA tensors (2-D,
        row-contiguous), w a uint8 CUDA tensor of N*K/blk blocks."""
        M, Kx = x.shape
        K = Kx if K is None else K
        N = c.shape[1] if N is None else N
        fn = lib().tcb_qgemm_act8 if act8 else lib().tcb_qgemm
        rc = fn(self._h, wtype, M, N, K, _ptr(w), _ptr(x), _dtype_code(x), x.stride(0), _ptr(c),
                _dtype_code(c), c.stride(0), int(bool(accumulate)), _stream(stream))
        self._check(rc, "tcb_qgemm_act8" if act8 else "tcb_qgemm")
        return c

    def qgemm_host(self, wtype, w, x, c, accumulate=False, stream=None):
        """tcb_qgemm_host: x and c torch CPU tensors (pinned or pageable, 2-D,
        row-contiguous), w a uint8 CUDA tensor.  With pinned c, read c after
        the stream synchronises."""
        M, K = x.shape
        N = c.shape[1]
        rc = lib().tcb_qgemm_host(self._h, wtype, M, N, K, _ptr(w), _ptr(x), _dtype_code(x), x.stride(0), _ptr(c),
                                  _dtype_code(c), c.stride(0), int(bool(accumulate)), _stream(stream))
        self._check(rc, "tcb_qgemm_host")
        return c

    def qgemm_act8(self, wtype, w, x, c, accumulate=True, stream=None):
        return self.qgemm(wtype, w, x, c, accumulate=accumulate, stream=stream, act8=True)

    def qdequant(self, wtype, w, n, out, stream=None):
        rc = lib().tcb_qdequant(self._h, wtype, _ptr(w), n, _ptr(out), _dtype_code(out), _stream(stream))
        self._check(rc, "tcb_qdequant")
        return out

    def qembed(self, wtype, w, V, D, idx, out, stream=None):
        import numpy as np

        ix = np.ascontiguousarray(idx, dtype=np.int64)
        rc = lib().tcb_qembed(self._h, wtype, _ptr(w), V, D, ix.ctypes.data, ix.size, _ptr(out), _stream(stream))
        self._check(rc, "tcb_qembed")
        return out

    def quant_upload(self, wtype, host, dev, stream=None) -> int:
        bad = ctypes.c_long(-1)
        rc = lib().tcb_quant_upload(self._h, wtype, _ptr(host), host.nbytes, _ptr(dev), ctypes.byref(bad),
                                    _stream(stream))
        if rc == 10:
            return bad.value
        self._check(rc, "tcb_quant_upload")
        return -1

    def quant_download(self, dev, host, stream=None):
        rc = lib().tcb_quant_download(self._h, _ptr(dev), host.nbytes, _ptr(host), _stream(stream))
        self._check(rc, "tcb_quant_download")
        return host

    def quant_zero(self, wtype, dev, nblocks, stream=None):
        rc = lib().tcb_quant_zero(self._h, wtype, _ptr(dev), nblocks, _stream(stream))
        self._check(rc, "tcb_quant_zero")
        return dev


def check_scales(wtype: int, host) -> int:
    """First block whose fp16 scale is NaN/Inf, or -1 (CheckQuantScales)."""
    bad = ctypes.c_long(-1)
    rc = lib().tcb_check_scales(wtype, _ptr(host), host.nbytes, ctypes.byref(bad))
    if rc not in (0, 10):
        raise TcbError(rc, "tcb_check_scales")
    return bad.value


STATIC_SCRATCH_BYTES = 4 << 20


def qgemm_act8_static(wtype, w, x, c, accumulate=True, stream=None):
    """tcb_qgemm_act8_static: Context.qgemm_act8 without a context, for
    callers that must not allocate device memory; its scratch is a fixed
    STATIC_SCRATCH_BYTES device array shared by all calls (order calls on
    one stream).  Runs on the current CUDA device."""
    M, K = x.shape
    N = c.shape[1]
    rc = lib().tcb_qgemm_act8_static(wtype, M, N, K, _ptr(w), _ptr(x), _dtype_code(x), x.stride(0), _ptr(c),
                                     _dtype_code(c), c.stride(0), int(bool(accumulate)), _stream(stream))
    if rc != 0:
        raise TcbError(rc, "tcb_qgemm_act8_static")
    return c
