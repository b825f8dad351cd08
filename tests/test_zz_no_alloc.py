"""tcb_qgemm_act8_static (the entry point that allocates no device memory)
against tcb_qgemm_act8 through the C ABI.  The int8-activation product is
bit-exact, so the two must agree bit for bit; two calls in a row check that
the shared static scratch carries nothing from one call into the next."""
import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import synth

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def case(wtype, M, N, K, seed):
    w = dev(synth.weight(wtype, N, K, seed))
    x = dev(synth.activations(M, K, seed + 1))
    return w, x


def test_static_matches_context_entry_two_calls():
    torch.cuda.set_device(0)
    ctx = T.Context(0)
    # second call smaller than the first, so stale scratch from call 1 sits
    # beyond and inside call 2's region
    for wtype, calls in ((T.Q4_K, [(4, 300, 2048), (3, 129, 1024)]),
                         (T.Q8_0, [(8, 257, 4096), (1, 64, 512)]),
                         (T.Q6_K, [(2, 96, 1536), (5, 33, 768)]),
                         (T.Q4_0, [(1, 4096, 4096), (6, 70, 2048)])):
        for i, (M, N, K) in enumerate(calls):
            w, x = case(wtype, M, N, K, 100 * wtype + i)
            want = torch.full((M, N), 0.25, dtype=torch.float32, device="cuda")
            got = want.clone()
            ctx.qgemm(wtype, w, x, want, act8=True, accumulate=True)
            rc = T.lib().tcb_qgemm_act8_static(wtype, M, N, K, w.data_ptr(), x.data_ptr(), T.F32, x.stride(0),
                                               got.data_ptr(), T.F32, got.stride(0), 1,
                                               torch.cuda.current_stream().cuda_stream)
            assert rc == 0, T.what_msg(rc)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (T.NAMES[wtype], M, N, K)


def test_static_set_and_16bit_out():
    ctx = T.Context(0)
    M, N, K = 3, 200, 2048
    w, x = case(T.Q4_K, M, N, K, 7)
    xb = x.to(torch.bfloat16)
    for _ in range(2):
        want = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        got = torch.empty_like(want)
        ctx.qgemm(T.Q4_K, w, xb, want, act8=True, accumulate=False)
        T.qgemm_act8_static(T.Q4_K, w, xb, got, accumulate=False)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_static_rejects_oversize():
    # 64 x 65536 activations need about 5.4 MB of scratch > 4 MiB
    M, N, K = 64, 8, 65536
    w = dev(synth.weight(T.Q4_K, N, K, 3))
    x = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    c = torch.full((M, N), 1.5, dtype=torch.float32, device="cuda")
    rc = T.lib().tcb_qgemm_act8_static(T.Q4_K, M, N, K, w.data_ptr(), x.data_ptr(), T.F32, K, c.data_ptr(), T.F32,
                                       N, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 11
    assert "static scratch" in T.what_msg(rc)
    torch.cuda.synchronize()
    assert bool((c == 1.5).all())


def test_static_allocates_no_device_memory():
    """After one call of each case (module and kernel loading, the runtime's
    own first-use costs), further calls leave the device's free memory
    unchanged."""
    shapes = [(T.Q4_K, 1, 64, 256), (T.Q8_0, 8, 257, 4096), (T.Q6_K, 5, 33, 768), (T.Q4_0, 60, 100, 8192)]
    cases = []
    for i, (wt, M, N, K) in enumerate(shapes):
        w, x = case(wt, M, N, K, 20 + i)
        cases.append((wt, w, x, torch.zeros((M, N), dtype=torch.float32, device="cuda")))
    for wt, w, x, c in cases:
        T.qgemm_act8_static(wt, w, x, c, accumulate=True)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        for wt, w, x, c in cases:
            T.qgemm_act8_static(wt, w, x, c, accumulate=True)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
