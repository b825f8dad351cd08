"""Batched greedy decode (tcb_llama_batch_*, TR's generate over a batch of
prompts, lib/layers.tr 712-770): several engines on the same weights, each
with its own prompt, K/V cache and position, stepped together.  Every
sequence's history is checked against the CPU reference (oracle/llama_ref.py)
fed that history -- logits within rel-L2 1e-3 at every step, every greedy
token the reference's -- and the tokens equal those of the engine stepped
alone; the captured batch graph replays the eager batch steps; prompts of
different lengths (positions differ inside one step), a prefilled batch, and
bad arguments."""
import os
import sys

import numpy as np
import pytest

import tcb_b200 as T
from tcb_b200 import llama

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from decoder_check import TOL, check_history, distinct_generated, rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=160, eps=1e-5, rope_theta=500000.0)
SEED = 15
GEN = 24


@pytest.fixture(scope="module")
def setup(oracle):
    host = llama.host_model(CFG, seed=SEED, varied=True)
    ctx = T.Context(0)
    dev = llama.device_model(CFG, SEED, host)
    rng = np.random.default_rng(41)
    # different lengths: the sequences sit at different positions in a step
    prompts = [rng.integers(0, CFG.vocab, n).astype(np.int64) for n in (8, 3, 13, 1, 8)]
    return ctx, host, dev, prompts


def run_batch(ctx, dev, prompts, steps, graph=False):
    engines = [llama.Llama(ctx, dev) for _ in prompts]
    for e, p in zip(engines, prompts):
        e.start(p)
    b = llama.Batch(engines)
    if graph:
        b.step(1)
        b.capture()
        for e, p in zip(engines, prompts):
            e.start(p)
    logits = []
    for _ in range(steps):
        b.step(1)
        logits.append(b.logits().copy())
    toks = [e.tokens(steps + 1) for e in engines]
    b.close()
    for e in engines:
        e.close()
    return toks, np.stack(logits, 1)  # [seq][step][vocab]


def test_batch_matches_reference(setup):
    ctx, host, dev, prompts = setup
    steps = max(len(p) for p in prompts) + GEN - 1
    toks, logits = run_batch(ctx, dev, prompts, steps)
    assert ctx.device_error() == 0
    for i, p in enumerate(prompts):
        assert list(toks[i][:len(p)]) == list(p)
        res = check_history(host, toks[i], len(p), {pos: logits[i][pos] for pos in range(steps)})
        assert res["checked_tokens"] == steps + 1 - len(p)
        assert res["checked_logits"] == steps
    assert sum(distinct_generated(t, len(p)) for t, p in zip(toks, prompts)) >= 16


def test_batch_equals_single_engines(setup):
    ctx, host, dev, prompts = setup
    steps = max(len(p) for p in prompts) + GEN - 1
    toks, logits = run_batch(ctx, dev, prompts, steps)
    for i, p in enumerate(prompts):
        m = llama.Llama(ctx, dev)
        m.start(p)
        for pos in range(steps):
            m.step(1)
            single = m.logits()
            # both are within TOL of the reference, but through different
            # kernels (the batch's multi-row products digitise x per 256
            # elements, the single step per 32), so they may differ by 2 TOL
            assert rel_l2(logits[i][pos], single) <= 2 * TOL, (i, pos)
            got, want = int(m.tokens(pos + 2)[pos + 1]), int(toks[i][pos + 1])
            if got != want:
                # the two kernels' roundings differ: only a tie may part them
                assert single[got] - single[want] < 2 * TOL * float(np.abs(single).max()), (i, pos)
                break
        m.close()


def test_batch_graph_replays_eager(setup):
    ctx, host, dev, prompts = setup
    steps = 20
    eager, _ = run_batch(ctx, dev, prompts, steps)
    graph, _ = run_batch(ctx, dev, prompts, steps, graph=True)
    for a, b in zip(eager, graph):
        assert list(a) == list(b)
    assert ctx.device_error() == 0


def test_batch_after_prefill(setup):
    """the batched prompt pass, then batched steps: every sequence's logits
    and tokens against the reference fed its history.  The plain test model
    (soft attention): its prompt pass stays within the float bound, as in
    tests/test_gpu_llama_prefill.py"""
    ctx = setup[0]
    host = llama.host_model(CFG, seed=7)
    dev = llama.device_model(CFG, 7, host)
    rng = np.random.default_rng(43)
    long = [rng.integers(0, CFG.vocab, n).astype(np.int64) for n in (70, 33, 90)]
    engines = [llama.Llama(ctx, dev) for _ in long]
    for e, p in zip(engines, long):
        e.start(p)
    llama.prefill_batch(engines)
    b = llama.Batch(engines)
    logits = []
    for _ in range(GEN):
        b.step(1)
        logits.append(b.logits().copy())
    got = [e.tokens(len(p) + GEN) for e, p in zip(engines, long)]
    b.close()
    for e in engines:
        e.close()
    for i, (p, t) in enumerate(zip(long, got)):
        lg = {len(p) - 1 + j: logits[j][i] for j in range(GEN)}
        res = check_history(host, t, len(p), lg)
        assert res["checked_tokens"] == GEN and res["checked_logits"] == GEN


def test_batch_bad_arguments(setup):
    ctx, host, dev, prompts = setup
    e = llama.Llama(ctx, dev)
    e.start(prompts[0])
    with pytest.raises(T.TcbError):
        llama.Batch([e, e])
    other = llama.device_model(llama.LlamaConfig(**{**CFG.__dict__, "n_layers": 1}), 3)
    f = llama.Llama(ctx, other)
    f.start(prompts[1])
    with pytest.raises(T.TcbError):
        llama.Batch([e, f])
    e.close()
    f.close()


def test_batch_long_rows_on_tensor_cores(setup):
    """a down projection of 9216-element rows: no multi-row matvec plan, so
    the batch step runs it on the tensor cores for all rows at once (fp16
    operands); every sequence's logits and tokens against the reference fed
    its history, on the plain test model"""
    ctx = setup[0]
    cfg = llama.LlamaConfig(n_layers=1, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=9216,
                            vocab=2048, max_ctx=64, eps=1e-5, rope_theta=500000.0)
    host = llama.host_model(cfg, seed=3)
    dev = llama.device_model(cfg, 3, host)
    rng = np.random.default_rng(47)
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.int64) for n in (5, 9, 2)]
    steps = 20
    toks, logits = run_batch(ctx, dev, prompts, steps)
    for i, p in enumerate(prompts):
        res = check_history(host, toks[i], len(p), {pos: logits[i][pos] for pos in range(steps)})
        assert res["checked_tokens"] == steps + 1 - len(p)
    assert ctx.device_error() == 0


def test_batch_graph_after_workspace_growth(setup):
    """A captured batch step keeps working after other calls on the context
    grow (and so move) its workspace: the batch owns the scratch of its
    products.  The down projection here runs on the tensor cores."""
    import torch

    from tcb_b200 import synth

    ctx = setup[0]
    cfg = llama.LlamaConfig(n_layers=1, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=9216,
                            vocab=2048, max_ctx=64, eps=1e-5, rope_theta=500000.0)
    host = llama.host_model(cfg, seed=3)
    dev = llama.device_model(cfg, 3, host)
    rng = np.random.default_rng(53)
    prompts = [rng.integers(0, cfg.vocab, n).astype(np.int64) for n in (4, 7)]
    eager, _ = run_batch(ctx, dev, prompts, 16)
    engines = [llama.Llama(ctx, dev) for _ in prompts]
    for e, p in zip(engines, prompts):
        e.start(p)
    b = llama.Batch(engines)
    b.step(1)
    b.capture()
    # a large product on the same context: its workspace grows
    w = torch.from_numpy(synth.weight(T.Q6_K, 4096, 8192, seed=5)).cuda()
    x = torch.randn((4096, 8192), device="cuda")
    y = torch.empty((4096, 4096), device="cuda")
    ctx.qgemm(T.Q6_K, w, x, y)
    torch.cuda.synchronize()
    for e, p in zip(engines, prompts):
        e.start(p)
    b.step(16)
    got = [e.tokens(17) for e in engines]
    b.close()
    for e in engines:
        e.close()
    for a_, b_ in zip(eager, got):
        assert list(a_) == list(b_)
    assert ctx.device_error() == 0


def test_batch16_on_tensor_cores(setup):
    """16 sequences: from 16 rows on every product of the batch step runs on
    the tensor cores (the weights streamed once for all rows, fp16 operands:
    about 2e-4 relative L2 per product, as in the prompt pass); each
    sequence's logits and tokens against the reference fed its history, on
    the plain test model, within 2e-3 (every product of every step, the head
    included, carries the fp16 rounding)"""
    ctx = setup[0]
    host = llama.host_model(CFG, seed=7)
    dev = llama.device_model(CFG, 7, host)
    rng = np.random.default_rng(59)
    prompts = [rng.integers(0, CFG.vocab, int(n)).astype(np.int64) for n in rng.integers(1, 12, 16)]
    steps = 24
    toks, logits = run_batch(ctx, dev, prompts, steps, graph=True)
    for i, p in enumerate(prompts):
        res = check_history(host, toks[i], len(p), {pos: logits[i][pos] for pos in range(1, steps)}, tol=2e-3)
        assert res["checked_tokens"] == steps + 1 - len(p)
    assert ctx.device_error() == 0
