"""A decoder loaded from a GGUF file (tcb_b200.llama_gguf: llama.cpp tensor
names, the converter's q/k row order, verbatim quantized blocks) decodes the
same greedy tokens on the GPU as the same weights handed over in memory, and
its first-step logits match bit for bit."""
import numpy as np
import pytest

import tcb_b200 as T
from tcb_b200 import llama, llama_gguf

pytestmark = pytest.mark.gpu

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=160, eps=1e-5, rope_theta=500000.0)
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)


def test_gguf_model_decodes_like_memory(tmp_path):
    host = llama.host_model(CFG, seed=9)
    path = str(tmp_path / "model.gguf")
    llama_gguf.write(path, CFG, host)
    cfg2, host2 = llama_gguf.load(path)
    # the file stores eps and theta as float32, which is what the engine uses
    cfg_mem = llama.LlamaConfig(**{**CFG.__dict__, "eps": cfg2.eps, "rope_theta": cfg2.rope_theta})
    ctx = T.Context(0)
    n = len(PROMPT) + 40
    outs = []
    for cfg, h in ((cfg_mem, host), (cfg2, host2)):
        m = llama.Llama(ctx, llama.device_model(cfg, 0, h))
        m.start(PROMPT)
        m.step(1)
        first = m.logits().copy()
        m.step(n - 2)
        outs.append((first, m.tokens(n)))
        m.close()
    assert np.array_equal(outs[0][0].view(np.uint32), outs[1][0].view(np.uint32))
    assert np.array_equal(outs[0][1], outs[1][1])


def test_mixed_types_decode_against_reference(tmp_path):
    """A llama.cpp Q4_K_M-like file (attn_v and ffn_down Q6_K in some layers,
    Q4_K in others; one layer's attn_output Q8_0): loaded from GGUF, its
    decode steps (q/k and v as two products where their types differ), the
    prompt pass and a batched step match the CPU reference fed the GPU's own
    history (decoder_check: logits within rel-L2 1e-3 at every step, tokens
    equal modulo float ties)."""
    import os
    import sys

    import torch

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from decoder_check import TOL, check_history

    cfg = llama.LlamaConfig(n_layers=3, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                            vocab=2048, max_ctx=96, eps=1e-5, rope_theta=500000.0)
    types = {"v": [T.Q6_K, T.Q4_K, T.Q6_K], "down": [T.Q6_K, T.Q4_K, T.Q4_K], "o": [T.Q6_K, T.Q8_0, T.Q6_K]}
    host = llama.host_model(cfg, seed=21, types=types)
    path = str(tmp_path / "mixed.gguf")
    llama_gguf.write(path, cfg, host)
    cfg2, host2 = llama_gguf.load(path)
    assert host2["types"] == types
    cfg2 = llama.LlamaConfig(**{**cfg2.__dict__, "max_ctx": cfg.max_ctx})
    ctx = T.Context(0)
    dev = llama.device_model(cfg2, 0, host2)
    gen = 16
    # eager steps: every step's logits
    m = llama.Llama(ctx, dev)
    m.start(PROMPT)
    logits = {}
    for pos in range(len(PROMPT) + gen - 1):
        m.step(1)
        logits[pos] = m.logits().copy()
    toks = m.tokens(len(PROMPT) + gen)
    m.close()
    res = check_history(host2, toks, len(PROMPT), logits)
    assert res["checked_logits"] == len(PROMPT) + gen - 1
    # the prompt pass, then steps: the reference's history again
    m = llama.Llama(ctx, dev)
    m.start(PROMPT)
    m.prefill()
    m.step(gen)
    check_history(host2, m.tokens(len(PROMPT) + gen), len(PROMPT))
    m.close()
    # a batched step over two sequences (the second prompt shifted)
    engines = [llama.Llama(ctx, dev) for _ in range(2)]
    prompts = [PROMPT, np.roll(PROMPT, 3)]
    for e, p in zip(engines, prompts):
        e.start(p)
    b = llama.Batch(engines)
    steps = len(PROMPT) + gen - 1
    blog = []
    for _ in range(steps):
        b.step(1)
        blog.append(b.logits().copy())
    torch.cuda.synchronize()
    for i, (e, p) in enumerate(zip(engines, prompts)):
        check_history(host2, e.tokens(steps + 1), len(p), {pos: blog[pos][i] for pos in range(steps)}, tol=2 * TOL)
    b.close()
    for e in engines:
        e.close()
    assert ctx.device_error() == 0
