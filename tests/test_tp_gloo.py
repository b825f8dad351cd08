"""The exchanges of the tensor-parallel decoder on two gloo ranks on the
CPU: rank 0's NCCL id reaches every rank (llama.share_id), and every rank's
64-byte peer handle reaches every rank in rank order (llama.gather_bytes)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from tcb_b200 import llama

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    got = llama.share_id(lambda: bytes(range(128)), rank)
    handles = llama.gather_bytes(bytes([rank]) * 64, world)
    q.put((rank, (got, handles)))
    dist.barrier()
    dist.destroy_process_group()


def test_share_id_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == res[1][0] == bytes(range(128))
    assert res[0][1] == res[1][1] == [bytes([0]) * 64, bytes([1]) * 64]
