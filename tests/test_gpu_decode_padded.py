"""A decoder whose Q6_K products take the row-padded copies, against the CPU
reference (oracle/llama_ref.py) fed the GPU's own history.

A 2-D TMA map needs a row stride that is a multiple of 16 bytes; a Q6_K row
of nb blocks is 210 * nb bytes, which is one only for nb a multiple of 8.
In this shape (d_model 512, ffn 2560, 4 query heads over 2 KV heads):
  * o (K = 512, 420-byte rows), the head (K = 512) and down (K = 2560,
    2100-byte rows: two TMA boxes per row) are read by the engine from copies
    with every row padded to a multiple of 16 bytes;
  * the attention heads of a KV head are spread over two CTAs.
Checked: every eager step's logits within rel-L2 1e-3 of the reference and
the greedy tokens equal to it (modulo float ties), the captured graph
equal to the eager steps with no extra launches, and a two-sequence batched
step (its products on the multi-row kernel over the same copies) against
the reference as well."""
import os
import sys

import numpy as np
import pytest
import torch

import tcb_b200 as T
from tcb_b200 import llama

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from decoder_check import TOL, check_history  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=2560,
                        vocab=2048, max_ctx=96, eps=1e-5, rope_theta=500000.0)
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)
GEN = 24


@pytest.fixture(scope="module")
def setup():
    host = llama.host_model(CFG, seed=23, varied=True)
    ctx = T.Context(0)
    return ctx, host, llama.device_model(CFG, 23, host)


def test_padded_q6k_rows_against_reference(setup):
    ctx, host, dev = setup
    n = len(PROMPT) + GEN
    m = llama.Llama(ctx, dev)
    m.start(PROMPT)
    logits = {}
    for pos in range(n - 1):
        m.step(1)
        logits[pos] = m.logits().copy()
    toks = m.tokens(n)
    m.close()
    res = check_history(host, toks, len(PROMPT), logits)
    assert res["checked_logits"] == n - 1 and res["checked_tokens"] == GEN
    # the captured graph repeats the eager steps
    g = llama.Llama(ctx, dev)
    g.start(PROMPT)
    g.capture()
    # the padded copies change no launch
    assert g.step_kernels() == 1 + 5 * CFG.n_layers + 4
    g.start(PROMPT)
    g.step(n - 1)
    assert list(g.tokens(n)) == list(toks)
    g.close()
    assert ctx.device_error() == 0


def test_padded_q6k_rows_batched(setup):
    ctx, host, dev = setup
    engines = [llama.Llama(ctx, dev) for _ in range(2)]
    prompts = [PROMPT, np.roll(PROMPT, 3)]
    for e, p in zip(engines, prompts):
        e.start(p)
    b = llama.Batch(engines)
    steps = len(PROMPT) + GEN - 1
    blog = []
    for _ in range(steps):
        b.step(1)
        blog.append(b.logits().copy())
    torch.cuda.synchronize()
    for i, (e, p) in enumerate(zip(engines, prompts)):
        check_history(host, e.tokens(steps + 1), len(p), {pos: blog[pos][i] for pos in range(steps)}, tol=2 * TOL)
    b.close()
    for e in engines:
        e.close()
    assert ctx.device_error() == 0
