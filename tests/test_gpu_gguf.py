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
