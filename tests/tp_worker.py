"""One rank of the tensor-parallel decoder checks (run with torchrun by
tests/test_gpu_tp.py).  Every run steps the engine one token at a time and
records, per step, the full logits (the ranks' vocabulary slices gathered
in rank order); rank 0 writes them with the token histories to an .npz.

    tp_worker.py OUT.npz steps            the small decoder (host model, the
                                          CPU reference's test model), greedy
    tp_worker.py OUT.npz prefill          the same, a 100-token prompt fed by
                                          the prompt pass
    tp_worker.py OUT.npz batch            the small decoder, five sequences of
                                          different lengths stepped together
                                          (tcb_llama_batch), eager and graph
    tp_worker.py OUT.npz shape70 [FORCED.npy]
                                          a 2-layer 70B-shaped decoder
                                          generated on the device (the same
                                          weights at every tensor-parallel
                                          degree), greedy, or fed the token
                                          history in FORCED.npy
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import tcb_b200 as T  # noqa: E402
from tcb_b200 import llama  # noqa: E402

CFG = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                        vocab=2048, max_ctx=160, eps=1e-5, rope_theta=500000.0)
SEED = 15
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)
LONG_PROMPT = np.random.default_rng(23).integers(0, CFG.vocab, 100).astype(np.int64)
GEN = {"steps": 64, "prefill": 40, "shape70": 40}

CFG70 = llama.LlamaConfig(n_layers=2, d_model=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn_dim=28672,
                          vocab=128256, max_ctx=96, eps=1e-5, rope_theta=500000.0)
SEED70 = 4
PROMPT70 = np.random.default_rng(29).integers(0, CFG70.vocab, 16).astype(np.int64)


def host_for(mode):
    """the host model of a mode: the varied decoder, the plain one for the
    prompt pass"""
    return llama.host_model(CFG, seed=7) if mode == "prefill" else llama.host_model(CFG, seed=SEED, varied=True)


def gathered_logits(m, world):
    lg = torch.from_numpy(m.logits().copy())
    parts = [None] * world
    dist.all_gather_object(parts, lg.numpy())
    return np.concatenate(parts)


BATCH_PROMPTS = [np.random.default_rng(41).integers(0, CFG.vocab, n).astype(np.int64) for n in (8, 3, 13, 1, 8)]
BATCH_STEPS = 36


def batch_main(ctx, rank, world, out_path, peer):
    host = llama.host_model(CFG, seed=SEED, varied=True)
    dev = llama.device_model(CFG, SEED, host, tp=(world, rank))
    engines = [llama.Llama(ctx, dev, tp=(world, rank)) for _ in BATCH_PROMPTS]
    # the residual rows summed by NCCL, or by the peer all-reduce (five
    # sequences fit its slots)
    engines[0].tp_init(llama.share_id(llama.nccl_unique_id, rank), peer=peer)
    runs = {}
    for mode in ("eager", "graph"):
        for e, p in zip(engines, BATCH_PROMPTS):
            e.start(p)
        b = llama.Batch(engines)
        if mode == "graph":
            b.step(1)
            b.capture()
            for e, p in zip(engines, BATCH_PROMPTS):
                e.start(p)
        logits = []
        for _ in range(BATCH_STEPS):
            b.step(1)
            lg = b.logits().copy()
            parts = [None] * world
            dist.all_gather_object(parts, lg)
            logits.append(np.concatenate(parts, axis=1))
        runs[mode] = ([e.tokens(BATCH_STEPS + 1) for e in engines], np.stack(logits, 1))
        b.close()
    all_tok = [None] * world
    dist.all_gather_object(all_tok, [t.tolist() for t in runs["eager"][0]])
    err = [None] * world
    dist.all_gather_object(err, ctx.device_error())
    if rank == 0:
        np.savez(out_path, eager=np.stack(runs["eager"][0]), graph=np.stack(runs["graph"][0]),
                 logits=runs["eager"][1], same_on_ranks=all(t == all_tok[0] for t in all_tok),
                 peer=bool(getattr(engines[0], "peer_active", False)),
                 device_errors=np.array(err, np.int64), first=0)
    for e in engines:
        e.close()
    dist.barrier()
    dist.destroy_process_group()


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    out_path, mode = sys.argv[1], sys.argv[2]
    ctx = T.Context(local)
    if mode in ("batch", "batch_peer"):
        return batch_main(ctx, rank, world, out_path, peer=mode == "batch_peer")
    if mode == "shape70":
        cfg = CFG70
        dev = llama.device_model(cfg, SEED70, tp=(world, rank), varied=True)
        forced = np.load(sys.argv[3]) if len(sys.argv) > 3 else None
        prompt = forced if forced is not None else PROMPT70
    else:
        cfg = CFG
        # the prompt pass on the plain model (its fp16 rounding stays within
        # the float bound there; tests/test_gpu_llama_prefill.py)
        host = host_for(mode)
        dev = llama.device_model(cfg, SEED, host, tp=(world, rank))
        forced = None
        prompt = LONG_PROMPT if mode == "prefill" else PROMPT
    gen = 0 if forced is not None else GEN[mode]
    n = len(prompt) + gen
    m = llama.Llama(ctx, dev, tp=(world, rank))
    m.tp_init(llama.share_id(llama.nccl_unique_id, rank))

    # eager, one step at a time, logits of every step
    m.start(prompt)
    first = 0
    if mode == "prefill":
        m.prefill()
        first = len(prompt) - 1
    logits = []
    for _ in range(first, n - 1):
        m.step(1)
        logits.append(gathered_logits(m, world))
    eager = m.tokens(n)
    # the captured graph
    m.start(prompt)
    m.capture()
    m.start(prompt)
    if mode == "prefill":
        m.prefill()
    m.step(n - 1 - first)
    graph = m.tokens(n)
    all_tok = [None] * world
    dist.all_gather_object(all_tok, eager.tolist())
    err = [None] * world
    dist.all_gather_object(err, ctx.device_error())
    if rank == 0:
        np.savez(out_path, eager=eager, graph=graph, logits=np.stack(logits), first=first,
                 same_on_ranks=all(t == all_tok[0] for t in all_tok), peer=bool(getattr(m, "peer_active", False)),
                 device_errors=np.array(err, np.int64))
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
