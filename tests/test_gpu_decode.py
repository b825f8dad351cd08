"""The Llama-shaped decoder (tcb_llama_*) against the CPU reference
(oracle/llama_ref.py, TR's GPT step over the oracle's float-path product):
first-step logits within the float tolerance, greedy tokens equal for 64
generated steps (a mismatch is accepted only where the reference's top-2
logit margin is below the logit tolerance, i.e. a tie at float precision),
and the captured CUDA graph reproducing the eager steps token for token."""
import numpy as np
import pytest

import tcb_b200 as T
from tcb_b200 import llama

pytestmark = pytest.mark.gpu

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=160, eps=1e-5, rope_theta=500000.0)
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)
GEN = 64


@pytest.fixture(scope="module")
def setup(oracle):
    from oracle.llama_ref import Reference

    host = llama.host_model(CFG, seed=5)
    ref_toks, ref_logits, margins = Reference(host).generate(PROMPT, len(PROMPT) + GEN - 1)
    ctx = T.Context(0)
    dev = llama.device_model(CFG, 5, host)
    return ctx, dev, ref_toks, ref_logits, margins


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def check_tokens(got, ref, ref_logits, margins):
    for i in range(1, len(ref)):
        if got[i] != ref[i]:
            tol = 1e-3 * float(np.abs(ref_logits[i - 1]).max())
            assert margins[i - 1] < tol, (i, got[i], ref[i], margins[i - 1], tol)
            return i  # a tie at float precision: the sequences part here
    return len(ref)


def test_first_step_logits(setup):
    ctx, dev, ref_toks, ref_logits, _ = setup
    m = llama.Llama(ctx, dev)
    m.start(PROMPT)
    m.step(1)
    assert rel_l2(m.logits(), ref_logits[0]) <= 1e-3
    for i in range(1, 6):
        m.step(1)
        assert rel_l2(m.logits(), ref_logits[i]) <= 1e-3, i
    m.close()


def test_greedy_tokens_eager_and_graph(setup):
    ctx, dev, ref_toks, ref_logits, margins = setup
    n = len(PROMPT) + GEN
    m = llama.Llama(ctx, dev)
    m.start(PROMPT)
    m.step(n - 1)
    eager = m.tokens(n)
    assert list(eager[:len(PROMPT)]) == list(PROMPT)
    matched = check_tokens(eager, ref_toks, ref_logits, margins)
    assert matched >= len(PROMPT) + 16
    # the captured graph replays the same step
    m.start(PROMPT)
    m.capture()
    m.start(PROMPT)
    m.step(n - 1)
    assert list(m.tokens(n)) == list(eager)
    m.close()


def test_bad_arguments(setup):
    ctx, dev, *_ = setup
    m = llama.Llama(ctx, dev)
    with pytest.raises(T.TcbError):
        m.start(np.array([CFG.vocab], np.int64))
    m.start(PROMPT)
    m.close()
