"""Host side of tensor parallelism on CPU: the handle exchange of
TensorParallel over a 2-rank gloo group (rank order, arbitrary bytes)."""
from __future__ import annotations

import os
import socket

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from conftest import load_pkg

    load_pkg()
    from minicpmo_b200.qwen3 import TensorParallel

    tp = TensorParallel(rank, world)
    got = tp.all_gather(bytes([rank]) * 64)
    barrier = tp.all_gather(b"")
    q.put((rank, [g[0] for g in got], [len(g) for g in got], barrier))
    dist.destroy_process_group()


def test_tensor_parallel_all_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, firsts, lens, barrier = q.get(timeout=120)
        out[rank] = (firsts, lens, barrier)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(2):
        firsts, lens, barrier = out[rank]
        assert firsts == [0, 1] and lens == [64, 64] and barrier == [b"", b""]
