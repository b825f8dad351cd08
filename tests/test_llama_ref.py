"""The CPU reference decoder (oracle/llama_ref.py) on the decoder tests'
"varied" model: its greedy continuation of the test prompt visits many
distinct tokens, with no top-2 margin inside the 1e-3 tie band, so the GPU
token-parity tests check attention over a growing context (a plain random
decoder repeats one token); and the host and device model generators agree
on the tensor-parallel slices (CPU only)."""
import os
import sys

import numpy as np

from tcb_b200 import llama

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from decoder_check import TOL, check_history, distinct_generated, min_margin_ratio  # noqa: E402

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=160, eps=1e-5, rope_theta=500000.0)
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)


def test_varied_model_continuation(oracle):
    from oracle.llama_ref import Reference

    host = llama.host_model(CFG, seed=15, varied=True)
    toks, logits, margins = Reference(host).generate(PROMPT, len(PROMPT) + 63)
    assert distinct_generated(toks, len(PROMPT)) >= 16
    assert min_margin_ratio(logits, margins, len(PROMPT)) > TOL
    # the checker accepts the reference's own history and rejects a changed token
    res = check_history(host, toks, len(PROMPT))
    assert res["checked_tokens"] == 64 and not res["ties"]
    bad = toks.copy()
    bad[len(PROMPT) + 10] = (bad[len(PROMPT) + 10] + 1) % CFG.vocab
    try:
        check_history(host, bad, len(PROMPT))
    except AssertionError:
        pass
    else:
        raise AssertionError("a wrong token passed the check")


def test_plain_model_is_degenerate(oracle):
    """The benchmark-distribution blocks collapse onto a couple of tokens:
    why the parity tests use the varied model."""
    from oracle.llama_ref import Reference

    host = llama.host_model(CFG, seed=5)
    toks, _, _ = Reference(host).generate(PROMPT, len(PROMPT) + 63)
    assert distinct_generated(toks, len(PROMPT)) <= 4
