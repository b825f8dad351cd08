"""CPU oracle pinned against TR's own golden vectors and known answers.

Mirrors internal/compute/tensor/quant_test.go and cpu_quant_q8_test.go of
sekerahmet/TCB.  No GPU needed.
"""
import json
import os
import struct

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "tr_golden.json")
FMT = {"q8_0": 8, "q4_0": 2, "q4_k": 12, "q6_k": 14}


def f16(v: float) -> int:
    return int(np.array([v], np.float16).view(np.uint16)[0])


def test_dequant_matches_llamacpp(oracle):
    """TestDequantMatchesLlamaCpp (quant_test.go:55-87): FNV-1a of the bits."""
    g = json.load(open(GOLDEN))
    for c in g["cases"]:
        fmt = FMT[c["format"]]
        y = oracle.dequant(fmt, oracle.random_quant(fmt, c["seed"], g["blocks"]))
        assert oracle.fnv1a_f32(y) == int(c["fnv1a64"], 16), c["format"]
        assert int(y.view(np.uint32)[c["at"]]) == int(c["sample_bits"], 16), c["format"]


def test_dequant_known_values(oracle):
    """TestDequantKnownValues (quant_test.go:89-137)."""
    two, half = 0x4000, 0x3800
    q8 = np.zeros(34, np.uint8)
    q8[0:2] = [two & 0xFF, two >> 8]
    q8[2], q8[3], q8[4] = 3, 0xFF, 0x80
    y = oracle.dequant(8, q8)
    assert list(y[:4]) == [6, -2, -256, 0]

    q4k = np.zeros(144, np.uint8)
    q4k[0:2] = [two & 0xFF, two >> 8]
    q4k[2:4] = [half & 0xFF, half >> 8]
    q4k[4], q4k[8] = 3, 4
    q4k[5], q4k[9] = 1, 2
    q4k[16] = 0x57
    y = oracle.dequant(12, q4k)
    assert y[0] == 2 * 3 * 7 - 0.5 * 4 and y[32] == 2 * 1 * 5 - 0.5 * 2 and y[1] == -2

    q40 = np.zeros(18, np.uint8)
    q40[0:2] = [two & 0xFF, two >> 8]
    q40[2], q40[3] = 0x3A, 0x08
    y = oracle.dequant(2, q40)
    assert (y[0], y[16], y[1], y[17], y[2]) == (4, -10, 0, -16, -16)
    z = oracle.zero_raw(2, 2)
    assert z[0] == 0 and z[1] == 0 and z[2] == 0x88 and z[17] == 0x88 and z[20] == 0x88
    assert not oracle.dequant(2, z).view(np.uint32).any()  # +0, never -0

    q6 = np.zeros(210, np.uint8)
    q6[208:210] = [two & 0xFF, two >> 8]
    q6[192] = 0xFD
    q6[0], q6[128] = 0x05, 0x02
    assert oracle.dequant(14, q6)[0] == 2 * -3 * (37 - 32)


def test_zero_scale_gives_zero(oracle):
    """TestDequantZeroScaleGivesZero (quant_test.go:140-163)."""
    for fmt, at in ((8, [0]), (2, [0]), (12, [0, 2]), (14, [208])):
        raw = np.full(oracle.BLOCK[fmt][1], 0x11, np.uint8)
        for a in at:
            raw[a:a + 2] = 0
        assert not oracle.dequant(fmt, raw).any()


def test_check_scales(oracle):
    """TestCheckQuantScales (quant_test.go:165-184)."""
    for fmt, at in ((8, 0), (2, 0), (12, 0), (12, 2), (14, 208)):
        size = oracle.BLOCK[fmt][1]
        assert oracle.check_scales(fmt, np.zeros(3 * size, np.uint8)) == -1
        for bad in (0x7E00, 0x7C00, 0xFC00):
            raw = np.zeros(3 * size, np.uint8)
            raw[size + at:size + at + 2] = [bad & 0xFF, bad >> 8]
            assert oracle.check_scales(fmt, raw) == 1


def test_f16_every_pattern(oracle):
    """IEEE half -> float for all 65536 patterns; NaN payload kept unquieted."""
    h = np.arange(1 << 16, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.lib().tcbo_f16_to_f32(int(v)) for v in h[::97]], np.float32)
    fin = np.isfinite(ref[::97])
    assert np.array_equal(got[fin].view(np.uint32), ref[::97][fin].view(np.uint32))
    nanbits = got[np.isnan(got)].view(np.uint32)
    srcbits = h[::97][np.isnan(ref[::97])].astype(np.uint32)
    # (a ctypes float return passes through a double, which quiets NaNs, so
    # compare the payload below the quiet bit)
    assert np.array_equal(nanbits & 0x3FFFFF, ((srcbits & 0x3FF) << 13) & 0x3FFFFF)


def test_nan_rule(oracle):
    """x86 NaN rule (gpu/kernel_quant.go:13-17): Q8 with an Inf scale and a
    zero code gives the default NaN; a NaN scale propagates quieted."""
    b = np.zeros(34, np.uint8)
    b[0:2] = [0x00, 0x7C]  # +Inf
    y = oracle.dequant(8, b)
    assert y.view(np.uint32)[0] == 0xFFC00000
    b[0:2] = [0x01, 0x7C]  # signalling NaN payload 1
    b[2] = 5
    y = oracle.dequant(8, b)
    assert y.view(np.uint32)[0] == (0x7F800000 | (1 << 13) | 0x400000)


@pytest.mark.parametrize("fmt,K", [(8, 32), (8, 576), (2, 64), (2, 1024), (12, 256), (12, 2560), (14, 512), (14, 3072)])
def test_quant_dot_matches_opened_dot(oracle, fmt, K):
    """TestQuantDotMatchesOpenedDot (cpu_quant_test.go:22-51): the dot is
    bit-identical to dequant + dotF32, for the AVX2 twin and the scalar one."""
    e, size = oracle.BLOCK[fmt]
    rng = np.random.default_rng(K)
    w = oracle.random_quant(fmt, K, 8 * K // e)
    x = rng.standard_normal(K).astype(np.float32)
    for n in range(8):
        row = w[n * K // e * size:(n + 1) * K // e * size]
        want = np.float32(oracle.dot_f32(x, oracle.dequant(fmt, row)))
        for scalar in (False, True):
            got = oracle.quant_dot(fmt, x, row, scalar=scalar)
            assert got.view(np.uint32) == want.view(np.uint32) or (np.isnan(got) and np.isnan(want))


def test_qgemm_float_independent_of_threads(oracle):
    """TestQuantMatMulIndependentOfWorkers (cpu_quant_test.go:173)."""
    rng = np.random.default_rng(3)
    N, K = 97, 512
    w = oracle.random_quant(12, 5, N * K // 256)
    a = rng.standard_normal((3, K)).astype(np.float32)
    one = oracle.qgemm_float(12, a, w, N, nthreads=1)
    many = oracle.qgemm_float(12, a, w, N, nthreads=7)
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))


def _q8_edge_blocks(blk):
    tiny = np.array([0x00400000], np.uint32).view(np.float32)[0]
    z = np.zeros(blk, np.float32)
    sat = np.where(np.arange(blk) % 2 == 0, 3.0, -3.0).astype(np.float32)
    big = np.full(blk, 1e-3, np.float32)
    big[5] = 1000
    small = np.zeros(blk, np.float32)
    small[0], small[1], small[2] = tiny, -tiny / 2, tiny / 4
    return [("zero", z, 0.0), ("sat", sat, np.float32(3) / np.float32(127)),
            ("big", big, np.float32(1000) / np.float32(127)), ("small", small, 0.0)]


@pytest.mark.parametrize("blk", [32, 256])
def test_quantize_q8_edge_blocks(oracle, blk):
    """TestQuantizeQ8KEdgeBlocks / TestQuantizeQ8BlockEdges
    (cpu_quant_q8_test.go:295-459)."""
    for name, x, d in _q8_edge_blocks(blk):
        q, dd, bs = oracle.quantize_q8(x, blk)
        assert dd[0] == np.float32(d), name
        if name == "sat":
            assert np.array_equal(q, np.where(np.arange(blk) % 2 == 0, 127, -127))
        elif name == "big":
            want = np.zeros(blk, np.int8)
            want[5] = 127
            assert np.array_equal(q, want)
        else:
            assert not q.any()
        assert np.array_equal(bs, q.reshape(-1, 16).astype(np.int16).sum(1).astype(np.int16))
    # two blocks: 0.5s round half-even 63.5 -> 64 (cpu_quant_q8_test.go:447-459)
    x = np.full(64, 0.5, np.float32)
    x[32:] = 1000
    x[0] = 1
    q, d, _ = oracle.quantize_q8(x, 32)
    assert d[0] == np.float32(1) / np.float32(127) and d[1] == np.float32(1000) / np.float32(127)
    assert q[0] == 127 and q[1] == 64 and q[32] == 127


def test_act8_rows_match_single_row(oracle):
    """Each output of the multi-row product is the one-row kernel's result,
    bit for bit (cpu_quant_q8_test.go:96-180)."""
    rng = np.random.default_rng(9)
    for fmt in (2, 8, 12, 14):
        e, size = oracle.BLOCK[fmt]
        N, K = 9, 512
        w = oracle.random_quant(fmt, 11 + fmt, N * K // e)
        a = rng.standard_normal((5, K)).astype(np.float32)
        many = oracle.qgemm_act8(fmt, a, w, N, nthreads=3)
        for m in range(5):
            one = oracle.qgemm_act8(fmt, a[m:m + 1], w, N, nthreads=1)
            assert np.array_equal(many[m].view(np.uint32), one[0].view(np.uint32))


def test_act8_keeps_non_finite(oracle):
    """TestQ8PathKeepsNonFinite (cpu_quant_q8_test.go:471-507): a row with
    NaN/Inf is the float path's own result; its neighbours are unaffected."""
    rng = np.random.default_rng(34)
    for fmt in (2, 12, 14):
        e, _ = oracle.BLOCK[fmt]
        N, K, M = 9, 512, 5
        w = oracle.random_quant(fmt, M + N, N * K // e)
        clean = rng.standard_normal((M, K)).astype(np.float32)
        for bad in (np.nan, np.inf, -np.inf):
            data = clean.copy()
            data[M // 2, K // 2] = bad
            got = oracle.qgemm_act8(fmt, data, w, N)
            want_clean = oracle.qgemm_act8(fmt, clean, w, N)
            want_bad = oracle.qgemm_float(fmt, data[M // 2:M // 2 + 1], w, N)
            for m in range(M):
                ref = want_bad[0] if m == M // 2 else want_clean[m]
                assert np.array_equal(got[m].view(np.uint32), ref.view(np.uint32))
        x = rng.standard_normal((M, K)).astype(np.float32)
        assert not np.array_equal(oracle.qgemm_float(fmt, x, w, N), oracle.qgemm_act8(fmt, x, w, N))


def test_act8_close_to_float(oracle):
    """The quantised product stays near the float one (scale of 2% of the
    norm, the bound cpu_quant_q8_test.go uses for its edge blocks)."""
    rng = np.random.default_rng(5)
    for fmt in (2, 8, 12, 14):
        e, _ = oracle.BLOCK[fmt]
        N, K = 64, 1024
        w = oracle.random_quant(fmt, 21, N * K // e)
        # small finite scales so the products stay finite
        y = oracle.dequant(fmt, w)
        if not np.all(np.isfinite(y)) or np.abs(y).max() > 1e4:
            continue
        a = rng.standard_normal((1, K)).astype(np.float32)
        f = oracle.qgemm_float(fmt, a, w, N)
        q = oracle.qgemm_act8(fmt, a, w, N)
        assert np.linalg.norm(f - q) <= 0.02 * np.linalg.norm(f) + 1e-30
