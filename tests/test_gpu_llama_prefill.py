"""The prompt pass of the decoder engine (tcb_llama_prefill): all but the last
prompt token fed as row batches through the tensor-core products and the
causal flash-attention kernel, then greedy steps.  Checked against the CPU
reference (oracle/llama_ref.py, TR's GPT step fed one token at a time) on the
"varied" test decoder, whose reference continuation visits many distinct
tokens with no top-2 margin inside the tolerance band: the logits of every
generated step within rel-L2 1e-3 and all greedy tokens equal to the
reference's, in one pass and in several (row batches that start off the
64-position tile grid, a last batch small enough for the non-tensor-core
product), for 2 and 4 query heads per KV head; the captured graph continues
from a prefilled cache exactly as the eager steps do; several engines fed in
one batched pass (tcb_llama_prefill_batch) give each one's own result."""
import os
import sys

import numpy as np
import pytest

import tcb_b200 as T
from tcb_b200 import llama

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from decoder_check import TOL, distinct_generated, min_margin_ratio, rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu

CFGS = {
    "gqa2": llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                              vocab=2048, max_ctx=512, eps=1e-5, rope_theta=500000.0),
    "gqa4": llama.LlamaConfig(n_layers=2, d_model=1024, n_heads=8, n_kv_heads=2, head_dim=128, ffn_dim=2048,
                              vocab=2048, max_ctx=512, eps=1e-5, rope_theta=500000.0),
}
NPROMPT = 300
GEN = 32
SEED = 10


@pytest.fixture(scope="module", params=sorted(CFGS))
def setup(request, oracle):
    from oracle.llama_ref import Reference

    cfg = CFGS[request.param]
    host = llama.host_model(cfg, seed=SEED, varied=True)
    prompt = np.random.default_rng(21).integers(0, cfg.vocab, NPROMPT).astype(np.int64)
    ref_toks, ref_logits, margins = Reference(host).generate(prompt, NPROMPT + GEN - 1)
    # a continuation worth checking: many distinct tokens, no tie at the tolerance
    assert distinct_generated(ref_toks, NPROMPT) >= 16
    assert min_margin_ratio(ref_logits, margins, NPROMPT) > TOL
    ctx = T.Context(0)
    dev = llama.device_model(cfg, SEED, host)
    return cfg, ctx, dev, prompt, ref_toks, ref_logits, margins


def run_prefill(ctx, dev, prompt, gen):
    """prefill, then gen eager steps one at a time: every step's logits and
    the token history"""
    m = llama.Llama(ctx, dev)
    m.start(prompt)
    m.prefill()
    logits = []
    for _ in range(gen):
        m.step(1)
        logits.append(m.logits().copy())
    toks = m.tokens(len(prompt) + gen)
    m.close()
    return logits, toks


def check_run(logits, toks, prompt, ref_toks, ref_logits):
    assert list(toks[:NPROMPT]) == list(prompt)
    for i, lg in enumerate(logits):
        assert rel_l2(lg, ref_logits[NPROMPT - 1 + i]) <= TOL, i
    assert list(toks) == list(ref_toks)


def test_prefill_against_reference(setup):
    cfg, ctx, dev, prompt, ref_toks, ref_logits, margins = setup
    logits, toks = run_prefill(ctx, dev, prompt, GEN)
    check_run(logits, toks, prompt, ref_toks, ref_logits)


def test_prefill_in_several_passes(setup, monkeypatch):
    cfg, ctx, dev, prompt, ref_toks, ref_logits, margins = setup
    # 80-row passes: batches start at positions 80, 160, 240 (off the 64-row
    # tile grid); the last has 59 rows (below the tensor-core path's minimum)
    monkeypatch.setenv("TCB_PREFILL_ROWS", "80")
    logits, toks = run_prefill(ctx, dev, prompt, GEN)
    check_run(logits, toks, prompt, ref_toks, ref_logits)


def test_prefill_then_graph(setup):
    cfg, ctx, dev, prompt, *_ = setup
    m = llama.Llama(ctx, dev)
    m.start(prompt)
    m.prefill()
    m.step(GEN)
    eager = m.tokens(NPROMPT + GEN)
    m.start(prompt)
    m.capture()
    m.start(prompt)
    m.prefill()
    m.step(GEN)
    assert list(m.tokens(NPROMPT + GEN)) == list(eager)
    m.close()


def test_prefill_state(setup):
    cfg, ctx, dev, prompt, ref_toks, *_ = setup
    m = llama.Llama(ctx, dev)
    # a one-token prompt has nothing to prefill
    m.start(prompt[:1])
    m.prefill()
    m.step(1)
    # after a step the cache already holds this sequence's positions
    with pytest.raises(T.TcbError):
        m.prefill()
    # a new start may prefill again; a short prompt takes the matvec path
    m.start(prompt[:5])
    m.prefill()
    m.step(1)
    m.close()


def test_prefill_batch(setup):
    """Several engines on the same model fed in one pass (the products over
    all their rows at once, attention per sequence): the same first-step
    logits as each fed alone, the reference's tokens for the full prompt."""
    cfg, ctx, dev, prompt, ref_toks, ref_logits, margins = setup
    prompts = [prompt, prompt[:150][::-1].copy(), prompt[40:117].copy(), prompt[:1].copy()]
    single = []
    for p in prompts:
        m = llama.Llama(ctx, dev)
        m.start(p)
        m.prefill()
        m.step(1)
        single.append(m.logits())
        m.close()
    engines = [llama.Llama(ctx, dev) for _ in prompts]
    for m, p in zip(engines, prompts):
        m.start(p)
    llama.prefill_batch(engines)
    for i, (m, p) in enumerate(zip(engines, prompts)):
        m.step(1)
        assert rel_l2(m.logits(), single[i]) <= 1e-4, i
    engines[0].step(GEN - 1)
    toks = engines[0].tokens(NPROMPT + GEN)
    assert list(toks) == list(ref_toks)
    # an engine that has stepped, or one given twice, is refused
    with pytest.raises(T.TcbError):
        llama.prefill_batch(engines[:2])
    engines[1].start(prompts[1])
    with pytest.raises(T.TcbError):
        llama.prefill_batch([engines[1], engines[1]])
    for m in engines:
        m.close()
