"""The Q4_K, Q6_K and Q4_0 float product of 2..16 activation rows in one weight
stream (tcb_mv_rows.cu) against the oracle's float path, through the C ABI.

TR's quantGemm with a few rows (tensor/cpu_quant.go:47-160): every row's
outputs within relative L2 1e-3 of TR's float path and within TR's GPU
max-abs bound (behavior_quant_test.go:283-302).  The cases cover 1..4 row
groups of the MMA (M 2..16, ragged M), ragged N, the BASELINE MLP shapes,
rows long enough that the activation digits are split over K ranges (the
split-K partials and their sum), accumulate and set, 16-bit activations and
outputs, strided views, NaN / Inf rows, determinism, and more than 16 rows
(row groups of 16, a last single row on the batch-1 kernel).  Q6_K rows
take this kernel when K is a multiple of 2048 (whole groups of 8
superblocks); other shapes keep the earlier kernels and are checked the same.
"""
import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
FMTS = [T.Q4_K, T.Q6_K, T.Q4_0]


@pytest.fixture(scope="module")
def ctx():
    return T.Context(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def rel_l2(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want.astype(np.float64)), 1e-30))


def check(got, want, K):
    assert rel_l2(got, want) <= REL_L2
    assert np.max(np.abs(got - want)) <= 1e-5 * np.sqrt(K) * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M", [2, 3, 4, 5, 8, 11, 12, 13, 16])
@pytest.mark.parametrize("NK", [(33, 256), (100, 2048), (257, 4096)])
def test_rows_match_oracle(ctx, oracle, fmt, M, NK):
    N, K = NK
    raw = synth.weight(fmt, N, K, seed=M + N)
    x = synth.activations(M, K, seed=M * 7 + N)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(fmt, x, raw, N), K)
    assert ctx.device_error() == 0


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M", [4, 8, 16])
@pytest.mark.parametrize("NK", [(11008, 4096), (4096, 11008)])
def test_rows_baseline_mlp_shapes(ctx, oracle, fmt, M, NK):
    """BASELINE config 2's shapes at batch 4/8 (and 16)."""
    N, K = NK
    raw = synth.weight(fmt, N, K, seed=3)
    x = synth.activations(M, K, seed=4)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(fmt, x, raw, N), K)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M", [5, 16])
@pytest.mark.parametrize("NK", [(512, 14336), (300, 28672), (4096, 8192)])
def test_rows_split_k(ctx, oracle, fmt, M, NK):
    """Rows whose digits do not fit one CTA beside its stages: the K ranges'
    partials are summed in range order (set and accumulate, and the same
    bits on a second call)."""
    N, K = NK
    raw = synth.weight(fmt, N, K, seed=N)
    x = synth.activations(M, K, seed=K)
    wd, xd = dev(raw), dev(x)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, wd, xd, c)
    got = host(c)
    check(got, oracle.qgemm_float(fmt, x, raw, N), K)
    c2 = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, wd, xd, c2)
    assert np.array_equal(host(c2).view(np.uint32), got.view(np.uint32))
    base = np.random.default_rng(1).standard_normal((M, N), dtype=np.float32)
    c3 = dev(base)
    ctx.qgemm(fmt, wd, xd, c3, accumulate=True)
    check(host(c3), oracle.qgemm_float(fmt, x, raw, N, c=base), K)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M", [17, 33, 40])
def test_rows_more_than_16(ctx, oracle, fmt, M):
    N, K = 200, 2048
    raw = synth.weight(fmt, N, K, seed=M)
    x = synth.activations(M, K, seed=M + 1)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(fmt, x, raw, N), K)


@pytest.mark.parametrize("fmt", FMTS)
def test_rows_16bit_and_views(ctx, oracle, fmt):
    """bf16 / f16 activations and outputs, strided rows, an activation view
    starting one element in (4-byte aligned), a slice of weight rows."""
    M, N, K = 6, 70, 2048
    raw = synth.weight(fmt, N, K, seed=9)
    xf = synth.activations(M, K + 1, seed=9)
    for xt in (torch.bfloat16, torch.float16):
        xd = dev(xf[:, :K]).to(xt)
        want = oracle.qgemm_float(fmt, xd.float().cpu().numpy(), raw, N)
        for ct in (torch.float32, torch.bfloat16, torch.float16):
            c = torch.zeros((M, N), dtype=ct, device="cuda")
            ctx.qgemm(fmt, dev(raw), xd, c)
            assert rel_l2(host(c), want) <= (1e-2 if ct != torch.float32 else REL_L2)
    xs = dev(xf)[:, 1:]
    c = torch.zeros((M, N + 5), dtype=torch.float32, device="cuda")[:, :N]
    ctx.qgemm(fmt, dev(raw), xs, c)
    check(host(c), oracle.qgemm_float(fmt, np.ascontiguousarray(xf[:, 1:]), raw, N), K)
    rb = K // 256 * (210 if fmt == T.Q6_K else 144)
    c2 = torch.zeros((M, 20), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw)[5 * rb:], dev(xf[:, :K]), c2)
    check(host(c2), oracle.qgemm_float(fmt, np.ascontiguousarray(xf[:, :K]), raw[5 * rb:25 * rb], 20), K)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("NK", [(100, 2048), (256, 14336)])
def test_rows_non_finite(ctx, oracle, fmt, NK):
    """A NaN or Inf in one row: TR's float path for the call, so NaN where
    TR has NaN and TR's values elsewhere in that row; the other rows within
    the float tolerance."""
    N, K = NK
    M = 7
    raw = synth.weight(fmt, N, K, seed=2)
    for bad in (np.nan, np.inf, -np.inf):
        x = synth.activations(M, K, seed=5)
        x[3, K // 3] = bad
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm(fmt, dev(raw), dev(x), c, accumulate=True)
        got, want = host(c), oracle.qgemm_float(fmt, x, raw, N)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        fin = ~np.isnan(want[3])
        assert np.array_equal(got[3][fin], want[3][fin])
        good = [m for m in range(M) if m != 3]
        check(got[good], want[good], K)
    # the next call with finite x is back on the integer path
    x = synth.activations(M, K, seed=6)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(fmt, x, raw, N), K)
    assert ctx.device_error() == 0
