"""The many-row product (prefill, M >= 64) on the tcgen05 tensor-core kernel,
checked against the CPU oracle through the C ABI.

TR's contract for the float path is the product of X with the opened
weights (quantGemm, tensor/cpu_quant.go:47-147; GPU bound
behavior_quant_test.go:283-302).  The tensor-core kernel rounds the
dequantised weights and the activations to fp16 (after exact power-of-two row
scaling) and accumulates in f32, so outputs are compared within the path's
stated relative-L2 bound of 1e-3.
"""
import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


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


def check(got, want, tol=REL_L2):
    assert np.isfinite(got).all()
    assert rel_l2(got, want) <= tol, rel_l2(got, want)
    # per row as well: a wrong tile cannot hide behind the others
    for m in range(0, got.shape[0], max(1, got.shape[0] // 16)):
        assert rel_l2(got[m], want[m]) <= 2 * tol, m


# (M, N, K): ragged M and N tiles, one and many superblocks, several tiles
SHAPES = [(64, 256, 256), (128, 512, 1024), (200, 300, 512), (130, 2000, 2304), (256, 1024, 4096)]


@pytest.mark.parametrize("MNK", SHAPES)
def test_tc_matches_oracle(ctx, oracle, MNK):
    M, N, K = MNK
    raw = synth.weight(T.Q4_K, N, K, seed=M + N)
    x = synth.activations(M, K, seed=K)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(T.Q4_K, x, raw, N))


def test_tc_lcg_blocks(ctx, oracle):
    """TR's seeded LCG blocks with small pinned scale exponents (every 6-bit
    scale and min pattern, all nibbles)."""
    M, N, K = 96, 272, 768
    raw = oracle.random_quant(T.Q4_K, 77, N * K // 256).reshape(-1, 144)
    raw[:, 1] = 0x1C | (raw[:, 1] & 0x83)
    raw[:, 3] = 0x1C | (raw[:, 3] & 0x83)
    raw = raw.reshape(-1)
    x = np.random.default_rng(3).standard_normal((M, K), dtype=np.float32)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(T.Q4_K, x, raw, N))


def test_tc_dtypes_strides_accumulate(ctx, oracle):
    """bf16/f16 activations and outputs, row strides, Gemm (+=) and GemmSet."""
    M, N, K = 160, 384, 1024
    raw = synth.weight(T.Q4_K, N, K, seed=5)
    xf = synth.activations(M, K + 8, seed=6)
    base = np.random.default_rng(7).standard_normal((M, N), dtype=np.float32)
    for xt in (torch.float32, torch.bfloat16, torch.float16):
        xd = dev(xf)[:, 3:3 + K].to(xt) if xt != torch.float32 else dev(xf)[:, 8:8 + K]
        xs = xd.float().cpu().numpy()
        for ct in (torch.float32, torch.bfloat16, torch.float16):
            tol = REL_L2 if ct == torch.float32 else 1e-2
            for acc in (False, True):
                cd = dev(base).to(ct)
                old = host(cd)
                ctx.qgemm(T.Q4_K, dev(raw), xd, cd, accumulate=acc)
                want = oracle.qgemm_float(T.Q4_K, xs, raw, N, c=old if acc else None)
                assert rel_l2(host(cd), want) <= tol, (xt, ct, acc)
    # strided output rows
    cw = torch.zeros((M, N + 40), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), dev(xf[:, :K]), cw[:, 20:20 + N])
    check(host(cw[:, 20:20 + N]), oracle.qgemm_float(T.Q4_K, xf[:, :K], raw, N))
    assert not host(cw[:, :20]).any() and not host(cw[:, 20 + N:]).any()


def test_tc_unaligned_activation_rows(ctx, oracle):
    """An activation view one element in (rows 4-byte, not 16-byte, aligned)
    and an odd row stride: the prep kernel's element-wise path."""
    M, N, K = 96, 256, 512
    raw = synth.weight(T.Q4_K, N, K, seed=21)
    xf = synth.activations(M, K + 3, seed=22)
    xd = dev(xf)[:, 1:1 + K]
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), xd, c)
    check(host(c), oracle.qgemm_float(T.Q4_K, xf[:, 1:1 + K], raw, N))


def test_tc_row_scales(ctx, oracle):
    """Rows of X and W far from unit scale: the power-of-two row scaling keeps
    fp16 in range (no Inf) and keeps precision for tiny rows."""
    M, N, K = 128, 256, 512
    raw = synth.weight(T.Q4_K, N, K, seed=11).reshape(N, K // 256, 144).copy()
    d = raw[:, :, 0:2].copy().view(np.float16)
    big = (np.abs(d) * np.float16(2048)).astype(np.float16)  # weights up to ~1e4 in rows 0..63
    raw[:64, :, 0:2] = big[:64].view(np.uint8)
    raw[64:128, :, 0:4] = (raw[64:128, :, 0:4].view(np.float16) * np.float16(1 / 4096)).astype(np.float16).view(np.uint8)
    raw = raw.reshape(-1)
    x = synth.activations(M, K, seed=12)
    x[:32] *= np.float32(3e4)
    x[32:64] *= np.float32(1e-6)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), dev(x), c)
    got, want = host(c), oracle.qgemm_float(T.Q4_K, x, raw, N)
    assert np.isfinite(got).all()
    # relative error per output row block (each block at its own scale)
    for r0 in range(0, M, 32):
        for n0 in range(0, N, 64):
            assert rel_l2(got[r0:r0 + 32, n0:n0 + 64], want[r0:r0 + 32, n0:n0 + 64]) <= REL_L2, (r0, n0)


def test_tc_non_finite_rows(ctx, oracle):
    """A NaN or Inf activation poisons its own output row only."""
    M, N, K = 64, 256, 512
    raw = synth.weight(T.Q4_K, N, K, seed=13)
    x = synth.activations(M, K, seed=14)
    x[5, 100] = np.nan
    x[9, 7] = np.inf
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), dev(x), c)
    got, want = host(c), oracle.qgemm_float(T.Q4_K, x, raw, N)
    assert np.isnan(got[5]).all() and np.isnan(want[5]).all()
    assert np.array_equal(np.isnan(got[9]), np.isnan(want[9]))
    assert np.array_equal(np.isposinf(got[9]), np.isposinf(want[9]))
    ok = np.ones(M, bool)
    ok[[5, 9]] = False
    check(got[ok], want[ok])


def test_tc_deterministic(ctx):
    M, N, K = 256, 512, 2048
    raw = dev(synth.weight(T.Q4_K, N, K, seed=15))
    x = dev(synth.activations(M, K, seed=16))
    outs = []
    for _ in range(3):
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        ctx.qgemm(T.Q4_K, raw, x, c)
        outs.append(host(c).view(np.uint32).copy())
    assert all(np.array_equal(o, outs[0]) for o in outs)


@pytest.mark.parametrize("NK", [(14336, 4096), (4096, 14336)])
def test_tc_prefill_config(ctx, oracle, NK):
    """The prefill configuration: Q4_K weights against bf16 activations,
    M = 2048.  The whole product runs on the GPU; 24 sampled rows are checked
    against the oracle (the full product is 1.2e11 multiply-adds)."""
    N, K = NK
    M = 2048
    raw = synth.weight(T.Q4_K, N, K, seed=N)
    xd = dev(synth.activations(M, K, seed=K)).to(torch.bfloat16)
    c = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, dev(raw), xd, c)
    rows = np.random.default_rng(1).choice(M, 24, replace=False)
    rows[:2] = [0, M - 1]
    xs = xd[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    got = host(c)[rows]
    check(got, oracle.qgemm_float(T.Q4_K, xs, raw, N))


# ---------------------------------------------------------------- other block types
# Q6_K, Q8_0, Q4_0 at M >= 64: the weights are dequantised exactly (TR's
# dequant) to row-scaled fp16 in workspace, then the same 2-CTA kernel runs
# with B loaded by TMA.

OTHER = [T.Q6_K, T.Q8_0, T.Q4_0]


@pytest.mark.parametrize("fmt", OTHER)
@pytest.mark.parametrize("MNK", [(64, 256, 256), (200, 300, 512), (130, 2000, 2304), (256, 1024, 4096)])
def test_tc_other_types(ctx, oracle, fmt, MNK):
    M, N, K = MNK
    raw = synth.weight(fmt, N, K, seed=M + N + fmt)
    x = synth.activations(M, K, seed=K + 1)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(fmt, dev(raw), dev(x), c)
    check(host(c), oracle.qgemm_float(fmt, x, raw, N))


@pytest.mark.parametrize("fmt", OTHER)
def test_tc_other_types_lcg_and_16bit(ctx, oracle, fmt):
    """TR's LCG blocks (small pinned scale exponents), bf16 activations, a
    bf16 output accumulated onto."""
    M, N, K = 96, 272, 768
    e, size = T.BLOCK[fmt]
    raw = oracle.random_quant(fmt, 55 + fmt, N * K // e).reshape(-1, size)
    for b in {T.Q8_0: [1], T.Q4_0: [1], T.Q6_K: [209]}[fmt]:
        raw[:, b] = 0x1C | (raw[:, b] & 0x83)
    raw = raw.reshape(-1)
    xd = dev(np.random.default_rng(fmt).standard_normal((M, K), dtype=np.float32)).to(torch.bfloat16)
    base = np.random.default_rng(2).standard_normal((M, N), dtype=np.float32)
    cd = dev(base).to(torch.bfloat16)
    old = host(cd)
    ctx.qgemm(fmt, dev(raw), xd, cd, accumulate=True)
    want = oracle.qgemm_float(fmt, xd.float().cpu().numpy(), raw, N, c=old)
    assert rel_l2(host(cd), want) <= 1e-2


def test_tc_q6k_down_projection(ctx, oracle):
    """The 8B decoder's down projection (Q6_K 4096 x 14336) at M = 2048,
    24 sampled rows against the oracle."""
    N, K, M = 4096, 14336, 2048
    raw = synth.weight(T.Q6_K, N, K, seed=3)
    xd = dev(synth.activations(M, K, seed=4)).to(torch.bfloat16)
    c = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q6_K, dev(raw), xd, c)
    rows = np.random.default_rng(5).choice(M, 24, replace=False)
    rows[:2] = [0, M - 1]
    xs = xd[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    check(host(c)[rows], oracle.qgemm_float(T.Q6_K, xs, raw, N))
