"""Tensor-parallel sharding of the decoder's block stores (CPU): every
rank's slices put back together give the full tensors, and the row-parallel
(K-split) products of the shards add up to the full product."""
import numpy as np
import pytest

from tcb_b200 import llama

CFG = llama.LlamaConfig(n_layers=1, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=32)


@pytest.fixture(scope="module")
def full():
    return llama.host_model(CFG, seed=3)


def blocks(a, kind, K):
    e, b = llama.BLOCK[llama.TYPES[kind]]
    return a.reshape(-1, K // e, b)


@pytest.mark.parametrize("tp", [2])
def test_shards_reassemble(full, tp):
    H, KVH, hd, D, F, V = CFG.n_heads, CFG.n_kv_heads, CFG.head_dim, CFG.d_model, CFG.ffn_dim, CFG.vocab
    parts = [llama.shard(CFG, full, tp, r) for r in range(tp)]
    h, kv, f = H // tp, KVH // tp, F // tp
    q = np.concatenate([blocks(p["qkv"][0], "qkv", D)[:h * hd] for p in parts])
    k = np.concatenate([blocks(p["qkv"][0], "qkv", D)[h * hd:(h + kv) * hd] for p in parts])
    v = np.concatenate([blocks(p["qkv"][0], "qkv", D)[(h + kv) * hd:] for p in parts])
    np.testing.assert_array_equal(np.concatenate([q, k, v]), blocks(full["qkv"][0], "qkv", D))
    o = np.concatenate([blocks(p["o"][0], "o", h * hd) for p in parts], axis=1)
    np.testing.assert_array_equal(o, blocks(full["o"][0], "o", H * hd))
    g = np.concatenate([blocks(p["gate_up"][0], "gate_up", D)[:f] for p in parts])
    u = np.concatenate([blocks(p["gate_up"][0], "gate_up", D)[f:] for p in parts])
    np.testing.assert_array_equal(np.concatenate([g, u]), blocks(full["gate_up"][0], "gate_up", D))
    d = np.concatenate([blocks(p["down"][0], "down", f) for p in parts], axis=1)
    np.testing.assert_array_equal(d, blocks(full["down"][0], "down", F))
    hd_ = np.concatenate([blocks(p["head"], "head", D) for p in parts])
    np.testing.assert_array_equal(hd_, blocks(full["head"], "head", D))
    for p in parts:
        assert p["tok_emb"] is full["tok_emb"] and p["attn_norm"] is full["attn_norm"]
        assert llama.local_shapes(CFG, tp)["o"] == (D, h * hd)


def test_row_parallel_products_add_up(full, oracle):
    tp, H, hd, D = 2, CFG.n_heads, CFG.head_dim, CFG.d_model
    x = np.random.default_rng(1).standard_normal(H * hd).astype(np.float32)
    want = oracle.qgemm_float(llama.TYPES["o"], x[None], full["o"][0], D)[0]
    got = np.zeros(D, np.float64)
    for r in range(tp):
        p = llama.shard(CFG, full, tp, r)
        xs = x[r * (H // tp) * hd:(r + 1) * (H // tp) * hd]
        got += oracle.qgemm_float(llama.TYPES["o"], xs[None], p["o"][0], D)[0]
    assert np.linalg.norm(got - want) <= 1e-5 * np.linalg.norm(want)
