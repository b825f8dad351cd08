"""The C ABI library loads and exports every entry point of include/tcb.h;
host-side checks behave as TR's backend does.  No GPU needed."""
import ctypes

import numpy as np
import pytest

import tcb_b200 as T
from tcb_b200 import synth


def test_library_exports_every_header_symbol():
    L = T.lib()
    syms = T.header_symbols()
    assert "tcb_qgemm" in syms and "tcb_qgemm_act8" in syms and len(syms) >= 13
    for s in syms:
        assert hasattr(L, s), s


def test_strerror_and_block_shape():
    for code in range(0, 11):
        assert T.lib().tcb_strerror(code)
    for w, (e, b) in T.BLOCK.items():
        ee, bb = ctypes.c_int(), ctypes.c_int()
        assert T.lib().tcb_block_shape(w, ctypes.byref(ee), ctypes.byref(bb)) == 0
        assert (ee.value, bb.value) == (e, b)
    assert T.lib().tcb_block_shape(3, None, None) == 2  # Q4_1: not on this path


def test_null_context_is_refused():
    L = T.lib()
    assert L.tcb_qgemm(None, T.Q4_K, 1, 1, 256, None, None, 0, 256, None, 0, 1, 1, None) == 1
    assert L.tcb_qgemm_act8(None, T.Q4_K, 1, 1, 256, None, None, 0, 256, None, 0, 1, 1, None) == 1
    assert L.tcb_qdequant(None, T.Q4_K, None, 256, None, 0, None) == 1
    assert L.tcb_llama_set_prefill_rows(None, 80) == 1
    assert L.tcb_qgemm_host(None, T.Q4_K, 1, 1, 256, None, None, 0, 256, None, 0, 1, 1, None) == 1


@pytest.mark.parametrize("w", [T.Q8_0, T.Q4_0, T.Q4_K, T.Q6_K])
def test_check_scales_matches_oracle(oracle, w):
    """CheckQuantScales (tensor/quant.go:108-128) on the host."""
    raw = oracle.random_quant(w, 7, 40)
    assert T.check_scales(w, raw) == -1 == oracle.check_scales(w, raw)
    at = {T.Q8_0: [0], T.Q4_0: [0], T.Q4_K: [0, 2], T.Q6_K: [208]}[w]
    for a in at:
        bad = raw.copy()
        off = 17 * T.BLOCK[w][1] + a
        bad[off:off + 2] = [0x00, 0x7C]
        assert T.check_scales(w, bad) == 17 == oracle.check_scales(w, bad)


def test_context_without_device_fails_gracefully():
    """TestNoDriverGraceful analogue: no GPU -> an error code, no crash."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = T.lib().tcb_ctx_create(0, ctypes.byref(h))
    assert rc == 5 and not h.value


def test_synth_q4k_scales_roundtrip(oracle):
    """The synthetic packer is the inverse of get_scale_min_k4."""
    rng = np.random.default_rng(1)
    sc = rng.integers(0, 64, (50, 8))
    m = rng.integers(0, 64, (50, 8))
    packed = synth.pack_q4k_scales(sc, m)
    blk = np.zeros((50, 144), np.uint8)
    blk[:, 0:2] = np.array([0x3C00], np.uint16).view(np.uint8)  # d = 1
    blk[:, 2:4] = np.array([0x3C00], np.uint16).view(np.uint8)  # dmin = 1
    blk[:, 4:16] = packed
    blk[:, 16:] = 0x11  # code 1 everywhere
    y = oracle.dequant(T.Q4_K, blk.reshape(-1)).reshape(50, 8, 32)
    assert np.array_equal(y[:, :, 0], (sc - m).astype(np.float32))
