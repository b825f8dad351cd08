"""Failure detection without a GPU fault: a bounded device-side wait that
runs out records TCB_ERR_TIMEOUT in the context's device error word, the
kernel returns, and the context stays usable.

The peer all-reduce of the tensor-parallel decoder (k_peer_ar) waits for
every other rank's values (each word carrying the call number).
tcb_peer_ar_selftest runs it as rank r of tp with every exchange buffer on
this device, so the other ranks' values never arrive (words that nothing
writes) and the wait gives up after a short poll limit; with one rank its
own values complete the wait.  A rank that leaves a real
tensor-parallel run is detected the same way on the remaining ranks.
"""
import time

import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import synth

pytestmark = pytest.mark.gpu

TIMEOUT = 7  # TCB_ERR_TIMEOUT


@pytest.fixture(scope="module")
def ctx():
    return T.Context(0)


def test_peer_wait_completes_with_its_own_values(ctx):
    ctx.device_error(clear=True)
    ctx.peer_ar_selftest(1, 0, 4096, 1 << 15)
    assert ctx.device_error() == 0


@pytest.mark.parametrize("tp,rank", [(2, 0), (2, 1), (8, 3)])
def test_peer_wait_gives_up_and_context_survives(ctx, oracle, tp, rank):
    ctx.device_error(clear=True)
    t0 = time.time()
    ctx.peer_ar_selftest(tp, rank, 8192, 1 << 14)
    elapsed = time.time() - t0
    assert ctx.device_error(clear=True) == TIMEOUT
    assert elapsed < 10.0
    assert ctx.device_error() == 0
    # the context still computes: a product against the oracle
    N, K, M = 64, 1024, 3
    raw = synth.weight(T.Q4_K, N, K, seed=4)
    x = synth.activations(M, K, seed=5)
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.qgemm(T.Q4_K, torch.from_numpy(raw).cuda(), torch.from_numpy(x).cuda(), c)
    torch.cuda.synchronize()
    want = oracle.qgemm_float(T.Q4_K, x, raw, N)
    got = c.cpu().numpy()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-3
    assert ctx.device_error() == 0


def test_selftest_rejects_bad_arguments(ctx):
    for args in [(0, 0, 4096), (9, 0, 4096), (2, 2, 4096), (2, 0, 4094)]:
        with pytest.raises(T.TcbError):
            ctx.peer_ar_selftest(*args, 100)
