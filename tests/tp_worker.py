"""One rank of the tensor-parallel decoder check (run with torchrun by
tests/test_gpu_tp.py): the small decoder sharded over the ranks, greedy
tokens eager and from the captured graph; with "prefill" a longer prompt fed
by the prompt pass (residual rows summed over the ranks).  Rank 0 prints the
tokens as JSON."""
import json
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
PROMPT = np.array([17, 901, 5, 1333, 42, 2047, 0, 777], np.int64)
LONG_PROMPT = np.random.default_rng(23).integers(0, CFG.vocab, 100).astype(np.int64)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    ctx = T.Context(local)
    host = llama.host_model(CFG, seed=5)
    dev = llama.device_model(CFG, 5, host, tp=(world, rank))
    m = llama.Llama(ctx, dev, tp=(world, rank))
    m.tp_init(llama.share_id(llama.nccl_unique_id, rank))
    gen = int(sys.argv[1] if len(sys.argv) > 1 else 64)
    pre = len(sys.argv) > 2 and sys.argv[2] == "prefill"
    prompt = LONG_PROMPT if pre else PROMPT
    n = len(prompt) + gen

    def feed():
        m.start(prompt)
        if pre:
            m.prefill()
            m.step(gen)
        else:
            m.step(n - 1)

    feed()
    eager = m.tokens(n)
    m.start(prompt)
    m.capture()
    feed()
    graph = m.tokens(n)
    all_tok = [None] * world
    dist.all_gather_object(all_tok, eager.tolist())
    if rank == 0:
        print(json.dumps({"eager": eager.tolist(), "graph": graph.tolist(), "same_on_ranks": all(t == all_tok[0] for t in all_tok)}))
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
