"""Parity of the sm_100a path with the CPU oracle, through the C ABI.

Mirrors TR's internal/compute/gpu/behavior_quant_test.go and the CPU
kernel tests: dequant bit-exact for every fp16 scale pattern, embedding
rows bit-exact, float products within the stated tolerance, the
int8-activation product bit-exact, determinism, error codes.
"""
import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import synth

pytestmark = pytest.mark.gpu

FORMATS = [T.Q8_0, T.Q4_0, T.Q4_K, T.Q6_K]
# float-accumulated outputs: relative L2 within 1e-3 (the path's stated bound)
REL_L2 = 1e-3


@pytest.fixture(scope="module")
def ctx():
    return T.Context(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def small_scale(oracle, fmt, seed, nblocks):
    """TR's smallScaleQuant (cpu_quant_test.go:71-88): LCG blocks whose fp16
    scales have their exponent pinned near 2^-8 so products stay finite."""
    raw = oracle.random_quant(fmt, seed, nblocks).reshape(nblocks, -1)
    for b in {T.Q8_0: [1], T.Q4_0: [1], T.Q4_K: [1, 3], T.Q6_K: [209]}[fmt]:
        raw[:, b] = 0x1C | (raw[:, b] & 0x83)
    return raw.reshape(-1)


def rel_l2(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want.astype(np.float64)), 1e-30))


def scale_offsets(fmt):
    return {T.Q8_0: [0], T.Q4_0: [0], T.Q4_K: [0, 2], T.Q6_K: [208]}[fmt]


# ---------------------------------------------------------------- dequant


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequant_every_scale_pattern(ctx, oracle, fmt):
    """TestQuantOpenMatchesCPUForEveryScale: all 65536 fp16 patterns,
    subnormal, Inf and NaN included, bit for bit."""
    e, size = T.BLOCK[fmt]
    pats = np.arange(1 << 16, dtype=np.uint16)
    for at in scale_offsets(fmt):
        raw = oracle.random_quant(fmt, 101 + at, pats.size).reshape(pats.size, size)
        raw[:, at:at + 2] = pats.view(np.uint8).reshape(-1, 2)
        raw = raw.reshape(-1)
        out = torch.empty(pats.size * e, dtype=torch.float32, device="cuda")
        ctx.qdequant(fmt, dev(raw), pats.size * e, out)
        want = oracle.dequant(fmt, raw)
        assert np.array_equal(host(out).view(np.uint32), want.view(np.uint32))


def test_dequant_q4k_both_scales_special(ctx, oracle):
    """TestQuantOpenQ4KBothScalesSpecial: the NaN rule of the subtraction."""
    special = [0, 0x8000, 1, 0x8001, 0x03FF, 0x7BFF, 0x7C00, 0xFC00, 0x7C01, 0xFC01, 0x7E00, 0xFE00, 0x7FFF, 0xFFFF]
    n = len(special) ** 2
    raw = oracle.random_quant(T.Q4_K, 3, n).reshape(n, 144)
    for i, a in enumerate(special):
        for j, b in enumerate(special):
            raw[i * len(special) + j, 0:2] = [a & 0xFF, a >> 8]
            raw[i * len(special) + j, 2:4] = [b & 0xFF, b >> 8]
    raw = raw.reshape(-1)
    out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
    ctx.qdequant(T.Q4_K, dev(raw), n * 256, out)
    assert np.array_equal(host(out).view(np.uint32), oracle.dequant(T.Q4_K, raw).view(np.uint32))


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequant_to_16_bit(ctx, oracle, fmt):
    """TestQuantOpenToOtherPrecisions: finite scales, f32 rounded once (RNE)."""
    e, _ = T.BLOCK[fmt]
    raw = small_scale(oracle, fmt, 4, 64)
    want = torch.from_numpy(oracle.dequant(fmt, raw))
    for dt in (torch.bfloat16, torch.float16):
        out = torch.empty(64 * e, dtype=dt, device="cuda")
        ctx.qdequant(fmt, dev(raw), 64 * e, out)
        assert torch.equal(out.cpu().view(torch.int16), want.to(dt).view(torch.int16))


@pytest.mark.parametrize("fmt", FORMATS)
def test_embedding_rows(ctx, oracle, fmt):
    """TestQuantEmbeddingOnTheCard: selected rows, bit for bit; bad index refused."""
    e, _ = T.BLOCK[fmt]
    V, D = 6, 2 * e
    raw = oracle.random_quant(fmt, 13, V * D // e)
    idx = [5, 0, 3, 3, 1, 2]
    out = torch.empty((len(idx), D), dtype=torch.float32, device="cuda")
    ctx.qembed(fmt, dev(raw), V, D, idx, out)
    assert np.array_equal(host(out).view(np.uint32), oracle.embedding(fmt, raw, D, idx).view(np.uint32))
    with pytest.raises(T.TcbError) as ei:
        ctx.qembed(fmt, dev(raw), V, D, [0, 6], out)
    assert ei.value.code == 9


@pytest.mark.parametrize("fmt", FORMATS)
def test_bytes_cross_unchanged(ctx, oracle, fmt):
    """Blocks go up and come back verbatim; a NaN/Inf scale is refused."""
    raw = oracle.random_quant(fmt, 17, 33)
    d = torch.empty(raw.size, dtype=torch.uint8, device="cuda")
    assert ctx.quant_upload(fmt, raw, d) == -1
    back = np.empty_like(raw)
    ctx.quant_download(d, back)
    assert np.array_equal(back, raw)
    bad = raw.copy()
    at = 5 * T.BLOCK[fmt][1] + scale_offsets(fmt)[0]
    bad[at:at + 2] = [0x00, 0xFC]
    assert ctx.quant_upload(fmt, bad, d) == 5


@pytest.mark.parametrize("fmt", FORMATS)
def test_zero_blocks(ctx, oracle, fmt):
    """QuantZeroRaw on the card: Q4_0 codes 0x88 (value +0, not -0); the
    opened zero blocks carry the same bits as TR's CPU dequant (Q6_K's
    (0*0)*(0-32) is -0 there too)."""
    e, size = T.BLOCK[fmt]
    d = torch.full((7 * size,), 0x5A, dtype=torch.uint8, device="cuda")
    ctx.quant_zero(fmt, d, 7)
    zero = oracle.zero_raw(fmt, 7)
    assert np.array_equal(host(d), zero)
    out = torch.empty(7 * e, dtype=torch.float32, device="cuda")
    ctx.qdequant(fmt, d, 7 * e, out)
    got = host(out)
    assert np.array_equal(got.view(np.uint32), oracle.dequant(fmt, zero).view(np.uint32))
    assert not got.any()
    if fmt == T.Q4_0:
        assert not got.view(np.uint32).any()


# ---------------------------------------------------------------- float path

SHAPES = [(1, 1), (7, 1), (9, 3), (16, 5), (33, 11), (70, 2), (300, 4)]  # (N, K in blocks)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M", [1, 2, 3, 8, 9, 17])
def test_qgemm_matches_oracle(ctx, oracle, fmt, M):
    """TestQuantGemvMatchesOpened / TestQuantMatMulRowsMatchOpened."""
    e, _ = T.BLOCK[fmt]
    rng = np.random.default_rng(M * 100 + fmt)
    for N, kb in SHAPES:
        K = kb * e
        raw = small_scale(oracle, fmt, N * 7 + kb, N * K // e)
        x = rng.standard_normal((M, K), dtype=np.float32)
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm(fmt, dev(raw), dev(x), c)
        want = oracle.qgemm_float(fmt, x, raw, N)
        got = host(c)
        assert rel_l2(got, want) <= REL_L2, (N, K)
        # TR's own GPU bound (behavior_quant_test.go:283-302), on the output scale
        assert np.max(np.abs(got - want)) <= 1e-5 * np.sqrt(K) * max(1.0, np.abs(want).max()), (N, K)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("kb,M", [(2, 3), (16, 8)])
def test_qgemm_precisions_and_views(ctx, oracle, fmt, kb, M):
    """TestQuantGemvShapesAndPrecisions: bf16/f16 x and c, row strides,
    an offset (unaligned) activation view, a slice of weight rows (with 16
    blocks per row every format's rows go through the multi-row launches)."""
    e, size = T.BLOCK[fmt]
    N, K = 6, kb * e
    raw = small_scale(oracle, fmt, 9, N * K // e)
    rng = np.random.default_rng(9)
    xf = rng.standard_normal((M, K + 1), dtype=np.float32)
    for xt in (torch.bfloat16, torch.float16):
        xd = dev(xf[:, :K]).to(xt)
        want = oracle.qgemm_float(fmt, xd.float().cpu().numpy(), raw, N)
        for ct in (torch.float32, torch.bfloat16, torch.float16):
            c = torch.zeros((M, N), dtype=ct, device="cuda")
            ctx.qgemm(fmt, dev(raw), xd, c)
            tol = 1e-2 if ct != torch.float32 else REL_L2
            assert rel_l2(c.float().cpu().numpy(), want) <= tol
    # strided rows and a view starting one element in (4-byte, not 16-byte, aligned)
    xs = dev(xf)[:, 1:]
    c = torch.zeros((M, N + 3), dtype=torch.float32, device="cuda")[:, :N]
    ctx.qgemm(fmt, dev(raw), xs, c)
    assert rel_l2(host(c), oracle.qgemm_float(fmt, xf[:, 1:], raw, N)) <= REL_L2
    # a slice of the weight's rows (offset on a block boundary)
    wd = dev(raw)
    c2 = torch.zeros((M, 3), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, wd[2 * (K // e) * size:], dev(xf[:, :K]), c2)
    assert rel_l2(host(c2), oracle.qgemm_float(fmt, xf[:, :K], raw[2 * (K // e) * size:5 * (K // e) * size], 3)) <= REL_L2


@pytest.mark.parametrize("fmt", FORMATS)
def test_qgemm_accumulates_and_sets(ctx, oracle, fmt):
    """TestQuantGemmAccumulates: Gemm adds to C, GemmSet overwrites it;
    K = 0 is the empty sum."""
    e, _ = T.BLOCK[fmt]
    N, K, M = 5, 2 * e, 4
    raw = small_scale(oracle, fmt, 11, N * K // e)
    rng = np.random.default_rng(11)
    x = rng.standard_normal((M, K), dtype=np.float32)
    base = rng.standard_normal((M, N), dtype=np.float32)
    c = dev(base)
    ctx.qgemm(fmt, dev(raw), dev(x), c, accumulate=True)
    assert rel_l2(host(c), oracle.qgemm_float(fmt, x, raw, N, c=base)) <= REL_L2
    c = dev(base)
    ctx.qgemm(fmt, dev(raw), dev(x), c, accumulate=False)
    assert rel_l2(host(c), oracle.qgemm_float(fmt, x, raw, N)) <= REL_L2
    c = dev(base)
    ctx.qgemm(fmt, dev(raw), dev(x[:, :0]), c, K=0, accumulate=True)
    assert np.array_equal(host(c), base)
    ctx.qgemm(fmt, dev(raw), dev(x[:, :0]), c, K=0, accumulate=False)
    assert not host(c).any()


@pytest.mark.parametrize("fmt", FORMATS)
def test_qgemm_deterministic(ctx, oracle, fmt):
    """TestQuantGemvIsDeterministic: the same bits every run."""
    e, _ = T.BLOCK[fmt]
    N, K = 40, 4 * e
    raw = dev(small_scale(oracle, fmt, 8, N * K // e))
    x = dev(np.random.default_rng(8).standard_normal((1, K), dtype=np.float32))
    outs = []
    for _ in range(3):
        c = torch.zeros((1, N), dtype=torch.float32, device="cuda")
        ctx.qgemm(fmt, raw, x, c)
        outs.append(host(c).view(np.uint32).copy())
    assert all(np.array_equal(o, outs[0]) for o in outs)


def test_qgemm_errors(ctx):
    """Refusals are status codes (TR panics with H6692 / H6695 analogues)."""
    w = torch.zeros(144 * 4, dtype=torch.uint8, device="cuda")
    x = torch.zeros((1, 256), dtype=torch.float32, device="cuda")
    c = torch.zeros((1, 4), dtype=torch.float32, device="cuda")
    L, h, s = T.lib(), ctx.handle, torch.cuda.current_stream().cuda_stream
    assert L.tcb_qgemm(h, 3, 1, 4, 256, w.data_ptr(), x.data_ptr(), 0, 256, c.data_ptr(), 0, 4, 1, s) == 2
    assert L.tcb_qgemm(h, T.Q4_K, 1, 4, 255, w.data_ptr(), x.data_ptr(), 0, 256, c.data_ptr(), 0, 4, 1, s) == 3
    assert L.tcb_qgemm(h, T.Q4_K, 1, 4, 256, w.data_ptr() + 1, x.data_ptr(), 0, 256, c.data_ptr(), 0, 4, 1, s) == 4
    assert L.tcb_qgemm(h, T.Q4_K, 1, 4, 256, w.data_ptr(), x.data_ptr(), 7, 256, c.data_ptr(), 0, 4, 1, s) == 2
    assert L.tcb_qgemm(h, T.Q4_K, 1, 4, 256, w.data_ptr(), x.data_ptr(), 0, 100, c.data_ptr(), 0, 4, 1, s) == 3
    assert L.tcb_qgemm(h, T.Q4_K, 1, 4, 256, None, x.data_ptr(), 0, 256, c.data_ptr(), 0, 4, 1, s) == 1


# ---------------------------------------------------------------- int8-activation path


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M", [1, 4, 5, 8, 17, 70])
def test_act8_bit_exact(ctx, oracle, fmt, M):
    """The int8-activation product equals TR's CPU kernels bit for bit
    (dotQ4Q8Go / dotQ4KQ8Go / dotQ6KQ8Go; Q8_0 by dotQ4Q8Go's fold)."""
    e, _ = T.BLOCK[fmt]
    rng = np.random.default_rng(M + fmt)
    for N, kb in [(1, 1), (9, 2), (33, 5), (64, 16), (130, 3)]:
        K = kb * e
        raw = small_scale(oracle, fmt, N + kb, N * K // e)
        x = rng.standard_normal((M, K), dtype=np.float32)
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm_act8(fmt, dev(raw), dev(x), c)
        assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(fmt, x, raw, N))), (N, K)


@pytest.mark.parametrize("fmt", FORMATS)
def test_act8_edge_blocks(ctx, oracle, fmt):
    """TestQuantizeQ8KEdgeBlocks / BlockEdges: zero, saturating, one large
    element, subnormal (127/amax overflows) blocks."""
    e, _ = T.BLOCK[fmt]
    tiny = np.array([0x00400000], np.uint32).view(np.float32)[0]
    rows = []
    r = np.zeros(e, np.float32); rows.append(r)
    rows.append(np.where(np.arange(e) % 2 == 0, 3.0, -3.0).astype(np.float32))
    r = np.full(e, 1e-3, np.float32); r[5] = 1000; rows.append(r)
    r = np.zeros(e, np.float32); r[0], r[1], r[2] = tiny, -tiny / 2, tiny / 4; rows.append(r)
    r = np.full(e, 0.5, np.float32); r[0] = 1; rows.append(r)  # 63.5 -> 64, half to even
    x = np.stack(rows)
    raw = small_scale(oracle, fmt, 77, 3)
    c = torch.zeros((x.shape[0], 3), dtype=torch.float32, device="cuda")
    ctx.qgemm_act8(fmt, dev(raw), dev(x), c)
    assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(fmt, x, raw, 3)))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("kb,M", [(2, 5), (16, 8)])
def test_act8_keeps_non_finite(ctx, oracle, fmt, kb, M):
    """TestQ8PathKeepsNonFinite: a row with NaN/Inf takes the float path
    (NaN/Inf where TR has them); the other rows stay bit-exact, also when
    they share a launch of several rows with it."""
    e, _ = T.BLOCK[fmt]
    N, K = 9, kb * e
    raw = small_scale(oracle, fmt, M + N, N * K // e)
    rng = np.random.default_rng(34)
    for bad in (np.nan, np.inf, -np.inf):
        x = rng.standard_normal((M, K), dtype=np.float32)
        x[M // 2, K // 2] = bad
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm_act8(fmt, dev(raw), dev(x), c)
        got, want = host(c), oracle.qgemm_act8(fmt, x, raw, N)
        for m in range(M):
            if m == M // 2:
                assert np.array_equal(np.isnan(got[m]), np.isnan(want[m]))
                fin = ~np.isnan(want[m])
                assert np.array_equal(got[m][fin], want[m][fin])  # +-Inf with the right sign
            else:
                assert np.array_equal(bits(got[m]), bits(want[m]))


# ---------------------------------------------------------------- benchmark shapes


def test_baseline_q8_0_4096_act8(ctx, oracle):
    """Config 0: Q8_0 4096x4096, x quantised on the fly: bit-exact."""
    raw = synth.weight(T.Q8_0, 4096, 4096, seed=1)
    x = synth.activations(1, 4096, seed=2)
    c = torch.zeros((1, 4096), dtype=torch.float32, device="cuda")
    ctx.qgemm_act8(T.Q8_0, dev(raw), dev(x), c)
    assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(T.Q8_0, x, raw, 4096)))


@pytest.mark.parametrize("fmt", [T.Q4_0, T.Q4_K])
@pytest.mark.parametrize("NK", [(11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("M", [1, 4, 8])
def test_baseline_mlp_shapes(ctx, oracle, fmt, NK, M):
    """Config 1: Q4_0 / Q4_K at Llama-7B MLP shapes, batch 1, 4, 8."""
    N, K = NK
    raw = synth.weight(fmt, N, K, seed=N + M)
    x = synth.activations(M, K, seed=M)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c)
    assert rel_l2(host(c), oracle.qgemm_float(fmt, x, raw, N)) <= REL_L2


# ---------------------------------------------------------------- tensor-core batch-1 path
# Rows whose byte length is a multiple of 16 take the TMA-staged int8 MMA
# kernel; these shapes cover several K ranges per tile (scratch combine),
# ragged last tiles, and one K range per tile (N above 8192 tiles).

FAST = [(1, 8), (17, 8), (70, 16), (130, 24), (300, 40)]  # (N, K in blocks)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("act8", [False, True])
def test_fast_path_matches_oracle(ctx, oracle, fmt, act8):
    e, _ = T.BLOCK[fmt]
    rng = np.random.default_rng(fmt * 7 + act8)
    for N, kb in FAST:
        K = kb * e
        raw = small_scale(oracle, fmt, N + kb, N * K // e)
        x = rng.standard_normal((1, K), dtype=np.float32)
        c = torch.zeros((1, N), dtype=torch.float32, device="cuda")
        ctx.qgemm(fmt, dev(raw), dev(x), c, act8=act8, accumulate=True)
        if act8:
            assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(fmt, x, raw, N))), (N, K)
        else:
            want = oracle.qgemm_float(fmt, x, raw, N)
            got = host(c)
            assert rel_l2(got, want) <= REL_L2, (N, K)
            assert np.max(np.abs(got - want)) <= 1e-5 * np.sqrt(K) * max(1.0, np.abs(want).max()), (N, K)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("act8", [False, True])
def test_fast_path_one_range_per_tile(ctx, oracle, fmt, act8):
    """More than 8192 tiles: every tile is one unit (no scratch combine)."""
    e, _ = T.BLOCK[fmt]
    N, K = 131088, 8 * e
    raw = synth.weight(fmt, N, K, seed=5)
    x = synth.activations(1, K, seed=6)
    c = torch.zeros((1, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c, act8=act8, accumulate=False)
    if act8:
        assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(fmt, x, raw, N)))
    else:
        assert rel_l2(host(c), oracle.qgemm_float(fmt, x, raw, N)) <= REL_L2


@pytest.mark.parametrize("fmt", FORMATS)
def test_fast_path_non_finite_x(ctx, oracle, fmt):
    """NaN/Inf in x: NaN where TR has NaN, the same signed Inf elsewhere."""
    e, _ = T.BLOCK[fmt]
    N, K = 40, 16 * e
    raw = small_scale(oracle, fmt, 3, N * K // e)
    for bad in (np.nan, np.inf, -np.inf):
        x = np.random.default_rng(1).standard_normal((1, K), dtype=np.float32)
        x[0, K // 3] = bad
        for act8 in (False, True):
            c = torch.zeros((1, N), dtype=torch.float32, device="cuda")
            ctx.qgemm(fmt, dev(raw), dev(x), c, act8=act8, accumulate=True)
            got, want = host(c), oracle.qgemm_float(fmt, x, raw, N)
            assert np.array_equal(np.isnan(got), np.isnan(want))
            fin = ~np.isnan(want)
            assert np.array_equal(got[fin], want[fin])


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M", [3, 8])
def test_fast_path_non_finite_rows(ctx, oracle, fmt, M):
    """Several rows of x, one with a NaN/Inf (the Q4_K kernel takes up to 8
    rows per launch): NaN where TR has NaN and the same values in that row,
    the other rows within the float tolerance."""
    e, _ = T.BLOCK[fmt]
    N, K = 40, 16 * e
    raw = small_scale(oracle, fmt, 5, N * K // e)
    for bad in (np.nan, np.inf):
        x = np.random.default_rng(2).standard_normal((M, K), dtype=np.float32)
        x[1, K // 3] = bad
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm(fmt, dev(raw), dev(x), c, accumulate=True)
        got, want = host(c), oracle.qgemm_float(fmt, x, raw, N)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        fin = ~np.isnan(want[1])
        assert np.array_equal(got[1][fin], want[1][fin])
        good = [m for m in range(M) if m != 1]
        assert rel_l2(got[good], want[good]) <= REL_L2


@pytest.mark.parametrize("NK", [(32768, 2560), (40000, 4096)])
def test_q6k_wide_kernel(ctx, oracle, NK):
    """Products of at least 32768 rows take the k-slot Q6_K kernel (a full
    and a ragged last tile, several staged chunks per row)."""
    N, K = NK
    raw = synth.weight(T.Q6_K, N, K, seed=N)
    x = synth.activations(1, K, seed=K)
    c = torch.zeros((1, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q6_K, dev(raw), dev(x), c, accumulate=True)
    want = oracle.qgemm_float(T.Q6_K, x, raw, N)
    got = host(c)
    assert rel_l2(got, want) <= REL_L2
    assert np.max(np.abs(got - want)) <= 1e-5 * np.sqrt(K) * max(1.0, np.abs(want).max())


def test_fast_path_mlp_shapes_16bit(ctx, oracle):
    """bf16 x and bf16/f16 c on the batch-1 kernel (one rounding of f32)."""
    N, K = 4096, 4096
    raw = synth.weight(T.Q4_K, N, K, seed=9)
    xd = dev(synth.activations(1, K, seed=10)).to(torch.bfloat16)
    want = oracle.qgemm_float(T.Q4_K, xd.float().cpu().numpy(), raw, N)
    for ct in (torch.float32, torch.bfloat16, torch.float16):
        c = torch.zeros((1, N), dtype=ct, device="cuda")
        ctx.qgemm(T.Q4_K, dev(raw), xd, c)
        assert rel_l2(c.float().cpu().numpy(), want) <= (REL_L2 if ct == torch.float32 else 1e-2)


# Q4_K partition over a fixed grid of 148 CTAs: (tile, block) units split
# evenly, tiles shared by neighbouring CTAs reduced through scratch counters.
PARTITION_SHAPES = [
    (32, 300),    # one tile over 300 blocks: every CTA holds a piece of it
    (40, 3),      # fewer units (6) than CTAs
    (1, 1),       # one unit
    (33, 37),     # two tiles, the second one row
    (4000, 5),    # many tiles, several per CTA, none split evenly
    (300, 16),    # tiles split at different blocks per CTA
]


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("accumulate", [False, True])
def test_q4k_partition(ctx, oracle, M, accumulate):
    rng = np.random.default_rng(M * 7 + accumulate)
    for N, kb in PARTITION_SHAPES:
        K = kb * 256
        raw = small_scale(oracle, T.Q4_K, N + kb, N * kb)
        x = rng.standard_normal((M, K), dtype=np.float32)
        base = rng.standard_normal((M, N), dtype=np.float32)
        want = oracle.qgemm_float(T.Q4_K, x, raw, N, c=base if accumulate else None)
        wd, xd = dev(raw), dev(x)
        outs = []
        for _ in range(3):  # the counters must be back at zero after every launch
            c = dev(base)
            ctx.qgemm(T.Q4_K, wd, xd, c, accumulate=accumulate)
            got = host(c)
            assert rel_l2(got, want) <= REL_L2, (N, K, M)
            outs.append(got.view(np.uint32).copy())
        assert all(np.array_equal(o, outs[0]) for o in outs), (N, K, M)
    assert ctx.device_error() == 0


# ---------------------------------------------------------------- int8 activations on the tensor cores


@pytest.mark.parametrize("M", [64, 129, 300])
def test_act8_tensor_cores_bit_exact(ctx, oracle, M):
    """Q4_K x Q8 activations from 64 rows on: the integer block sums on
    tcgen05 (kind::i8), the fold in TR's order -- bit for bit TR's
    quantGemmQ8 (cpu_quant_q8.go:186-259), on ragged tiles of activation
    rows (128) and weight rows (64), GemmSet and Gemm."""
    rng = np.random.default_rng(M)
    for N, kb in [(64, 1), (100, 4), (257, 16)]:
        K = kb * 256
        raw = small_scale(oracle, T.Q4_K, N + kb + M, N * kb)
        x = rng.standard_normal((M, K), dtype=np.float32)
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm_act8(T.Q4_K, dev(raw), dev(x), c)
        assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(T.Q4_K, x, raw, N))), (N, K)
        base = rng.standard_normal((M, N), dtype=np.float32)
        c = dev(base)
        ctx.qgemm_act8(T.Q4_K, dev(raw), dev(x), c, accumulate=True)
        assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(T.Q4_K, x, raw, N, c=base))), (N, K)
    assert ctx.device_error() == 0


def test_act8_tensor_cores_inputs_and_non_finite(ctx, oracle):
    """bf16 and f16 activations, strided rows, BASELINE-distribution blocks
    (every fp16 scale |N(0, 0.01)|), and rows holding NaN / Inf (TR's float
    path for those rows only)."""
    M, N, K = 96, 192, 4096
    raw = synth.weight(T.Q4_K, N, K, seed=12)
    rng = np.random.default_rng(12)
    xf = rng.standard_normal((M, K + 8), dtype=np.float32)
    for xt in (torch.bfloat16, torch.float16):
        xd = dev(xf[:, :K]).to(xt)
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm_act8(T.Q4_K, dev(raw), xd, c)
        want = oracle.qgemm_act8(T.Q4_K, xd.float().cpu().numpy(), raw, N)
        assert np.array_equal(bits(host(c)), bits(want))
    xs = dev(xf)[:, 4:4 + K]  # row stride K + 8, 16-byte offset
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm_act8(T.Q4_K, dev(raw), xs, c)
    assert np.array_equal(bits(host(c)), bits(oracle.qgemm_act8(T.Q4_K, np.ascontiguousarray(xf[:, 4:4 + K]), raw, N)))
    x = xf[:, :K].copy()
    x[3, 100] = np.nan
    x[70, 4000] = np.inf
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm_act8(T.Q4_K, dev(raw), dev(x), c)
    got, want = host(c), oracle.qgemm_act8(T.Q4_K, x, raw, N)
    for m in range(M):
        if m in (3, 70):
            assert np.array_equal(np.isnan(got[m]), np.isnan(want[m]))
            fin = ~np.isnan(want[m])
            assert np.array_equal(got[m][fin], want[m][fin])
        else:
            assert np.array_equal(bits(got[m]), bits(want[m])), m
    assert ctx.device_error() == 0


def test_act8_tensor_cores_prefill_rows(ctx, oracle):
    """BASELINE config 4's product (Q4_K 14336 x 4096) with 2048 activation
    rows through the tensor-core kernel; rows spread over the launch checked
    bit for bit against the oracle (the full product takes the CPU minutes)."""
    N, K, M = 14336, 4096, 2048
    raw = synth.weight(T.Q4_K, N, K, seed=21)
    x = synth.activations(M, K, seed=22)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm_act8(T.Q4_K, dev(raw), dev(x), c)
    got = host(c)
    rows = [0, 1, 127, 128, 1000, 2047]
    want = oracle.qgemm_act8(T.Q4_K, x[rows], raw, N)
    assert np.array_equal(bits(got[rows]), bits(want))
    assert ctx.device_error() == 0
