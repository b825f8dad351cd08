"""tcb_qgemm_host: the product over host buffers gives tcb_qgemm's results
bit for bit, for every placement of x and c (pinned host memory, which the
kernels read and write in place; pageable host memory, copied through the
context's device buffers; device memory), both output modes (set and
accumulate), 16-bit activations and outputs, strided rows, the batch-1,
few-row and tensor-core paths, and calls issued back to back on one stream
(the staged x of one call is not overwritten while the previous product
still reads it)."""
import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    return T.Context(0)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


def reference(ctx, fmt, wd, x, base, accumulate):
    """tcb_qgemm on device copies of x and c."""
    xd = x.cuda()
    cd = base.cuda()
    ctx.qgemm(fmt, wd, xd, cd, accumulate=accumulate)
    torch.cuda.synchronize()
    return cd.cpu()


def host_tensor(t, pinned):
    return t.clone().pin_memory() if pinned else t.clone()


@pytest.mark.parametrize("fmt", [T.Q4_K, T.Q6_K, T.Q4_0, T.Q8_0])
@pytest.mark.parametrize("M", [1, 5, 70])
@pytest.mark.parametrize("where", ["pinned", "pageable", "pinned_x", "pinned_c", "device_x"])
def test_host_buffers_match_device_call(ctx, fmt, M, where):
    N, K = 300, 2048
    wd = torch.from_numpy(synth.weight(fmt, N, K, seed=M + fmt)).cuda()
    x = torch.from_numpy(synth.activations(M, K, seed=M))
    base = torch.from_numpy(np.random.default_rng(M).standard_normal((M, N), dtype=np.float32))
    for accumulate in (False, True):
        want = reference(ctx, fmt, wd, x, base, accumulate)
        xh = x.cuda() if where == "device_x" else host_tensor(x, where in ("pinned", "pinned_x"))
        ch = host_tensor(base, where in ("pinned", "pinned_c", "device_x"))
        ctx.qgemm_host(fmt, wd, xh, ch, accumulate=accumulate)
        torch.cuda.synchronize()
        assert np.array_equal(bits(ch.numpy()), bits(want.numpy())), (where, accumulate)
    assert ctx.device_error() == 0


@pytest.mark.parametrize("pinned", [True, False])
def test_host_16bit_and_strided_rows(ctx, pinned):
    M, N, K = 6, 200, 4096
    wd = torch.from_numpy(synth.weight(T.Q4_K, N, K, seed=3)).cuda()
    wide = torch.from_numpy(synth.activations(M, K + 8, seed=4)).to(torch.bfloat16)
    x = host_tensor(wide, pinned)[:, 4:K + 4]  # row stride K + 8, 8-byte offset
    for ct in (torch.float32, torch.float16):
        want = torch.zeros((M, N), dtype=ct, device="cuda")
        ctx.qgemm(T.Q4_K, wd, x.cuda(), want)
        cwide = host_tensor(torch.zeros((M, N + 5), dtype=ct), pinned)
        c = cwide[:, :N]
        ctx.qgemm_host(T.Q4_K, wd, x, c)
        torch.cuda.synchronize()
        assert np.array_equal(bits(c.numpy()), bits(want.cpu().numpy()))
        assert not cwide[:, N:].any()  # the row padding is left alone


def test_host_calls_back_to_back(ctx):
    """Eight calls on one stream without a synchronisation between them, each
    with its own x and c: every result is its own x's product."""
    N, K = 11008, 4096
    wd = torch.from_numpy(synth.weight(T.Q4_K, N, K, seed=5)).cuda()
    xs = [torch.from_numpy(synth.activations(1, K, seed=10 + i)).pin_memory() for i in range(8)]
    cs = [torch.zeros((1, N), dtype=torch.float32).pin_memory() for _ in range(8)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for x, c in zip(xs, cs):
            ctx.qgemm_host(T.Q4_K, wd, x, c, stream=s)
    s.synchronize()
    for x, c in zip(xs, cs):
        want = reference(ctx, T.Q4_K, wd, x, torch.zeros((1, N)), False)
        assert np.array_equal(bits(c.numpy()), bits(want.numpy()))


def test_host_argument_errors(ctx):
    L = T.lib()
    x = torch.zeros((1, 256)).pin_memory()
    c = torch.zeros((1, 4)).pin_memory()
    wd = torch.zeros(4 * 144, dtype=torch.uint8, device="cuda")
    assert L.tcb_qgemm_host(None, T.Q4_K, 1, 4, 256, wd.data_ptr(), x.data_ptr(), T.F32, 256, c.data_ptr(), T.F32,
                            4, 0, None) == 1
    assert L.tcb_qgemm_host(ctx._h, 3, 1, 4, 256, wd.data_ptr(), x.data_ptr(), T.F32, 256, c.data_ptr(), T.F32,
                            4, 0, None) == 2
    assert L.tcb_qgemm_host(ctx._h, T.Q4_K, 1, 4, 100, wd.data_ptr(), x.data_ptr(), T.F32, 256, c.data_ptr(), T.F32,
                            4, 0, None) == 3
