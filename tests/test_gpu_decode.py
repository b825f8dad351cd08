"""The Llama-shaped decoder (tcb_llama_*) against the CPU reference
(oracle/llama_ref.py, TR's GPT step over the oracle's float-path product;
TR lib/layers.tr GPT.single_step 658-666, generate 712-770).

The test model is the "varied" decoder (tcb_b200/llama.py): its reference
greedy continuation of the prompt visits many distinct tokens, so the 64
steps exercise attention over a growing context rather than a fixed point.

  * 64 greedy steps: at every step the logits are within rel-L2 1e-3 of the
    reference fed the GPU's own history, and every generated token is the
    reference's greedy token.  The model's reference continuation has no
    top-2 margin inside the tolerance band (asserted), so the tokens must
    equal the reference's own greedy continuation, all 64 of them.
  * teacher forcing: a random 64-token continuation fed as prompt, logits
    compared at every position.
  * the captured CUDA graph reproduces the eager steps token for token."""
import os
import sys

import numpy as np
import pytest

import tcb_b200 as T
from tcb_b200 import llama

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from decoder_check import TOL, check_history, distinct_generated, min_margin_ratio, rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=160, eps=1e-5, rope_theta=500000.0)
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)
GEN = 64
SEED = 15
MIN_DISTINCT = 16


@pytest.fixture(scope="module")
def setup(oracle):
    from oracle.llama_ref import Reference

    host = llama.host_model(CFG, seed=SEED, varied=True)
    ref_toks, ref_logits, margins = Reference(host).generate(PROMPT, len(PROMPT) + GEN - 1)
    ctx = T.Context(0)
    dev = llama.device_model(CFG, SEED, host)
    return ctx, host, dev, ref_toks, ref_logits, margins


def run_steps(ctx, dev, prompt, nsteps):
    """Eager steps one at a time: the token history and every step's logits."""
    m = llama.Llama(ctx, dev)
    m.start(prompt)
    logits = {}
    for pos in range(nsteps):
        m.step(1)
        logits[pos] = m.logits().copy()
    toks = m.tokens(nsteps + 1)
    m.close()
    return toks, logits


def test_reference_continuation_is_varied(setup):
    _, _, _, ref_toks, ref_logits, margins = setup
    assert distinct_generated(ref_toks, len(PROMPT)) >= MIN_DISTINCT
    # no reference greedy pick is a tie at the tolerance: the GPU must match all 64
    assert min_margin_ratio(ref_logits, margins, len(PROMPT)) > TOL


def test_greedy_64_steps(setup):
    ctx, host, dev, ref_toks, ref_logits, _ = setup
    n = len(PROMPT) + GEN
    toks, logits = run_steps(ctx, dev, PROMPT, n - 1)
    assert list(toks[:len(PROMPT)]) == list(PROMPT)
    assert list(toks) == list(ref_toks)
    res = check_history(host, toks, len(PROMPT), logits)
    assert res["checked_tokens"] == GEN and res["checked_logits"] == n - 1 and not res["ties"]
    # the logits of the reference's own run agree at every step as well
    for pos in range(n - 1):
        assert rel_l2(logits[pos], ref_logits[pos]) <= TOL, pos


def test_teacher_forced_logits(setup):
    ctx, host, dev, *_ = setup
    rng = np.random.default_rng(31)
    forced = np.concatenate([PROMPT, rng.integers(0, CFG.vocab, GEN)]).astype(np.int64)
    toks, logits = run_steps(ctx, dev, forced, len(forced) - 1)
    assert list(toks) == list(forced)
    res = check_history(host, forced, len(forced), logits)
    assert res["checked_logits"] == len(forced) - 1


def test_graph_replays_eager(setup):
    ctx, host, dev, ref_toks, *_ = setup
    n = len(PROMPT) + GEN
    m = llama.Llama(ctx, dev)
    m.start(PROMPT)
    m.step(n - 1)
    eager = m.tokens(n)
    assert list(eager) == list(ref_toks)
    m.start(PROMPT)
    m.capture()
    # embedding; per layer qkv (RMSNorm fused), attention, o, gate_up (RMSNorm
    # and SwiGLU fused), down; final RMSNorm, head, the two-level greedy pick
    assert m.step_kernels() == 1 + 5 * CFG.n_layers + 4
    m.start(PROMPT)
    m.step(n - 1)
    assert list(m.tokens(n)) == list(eager)
    m.close()


def test_bad_arguments(setup):
    ctx, host, dev, *_ = setup
    m = llama.Llama(ctx, dev)
    with pytest.raises(T.TcbError):
        m.start(np.array([CFG.vocab], np.int64))
    m.start(PROMPT)
    m.close()
