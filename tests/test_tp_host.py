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


# --------------------------------------------------------------------------
# The fused exchange protocol (minicpm-o-uya_b200/csrc/tp_proto.h) on host
# threads: every rank's partial summed in rank order, no slot overwritten
# while a slower rank still reads it, and a rank that leaves between steps
# makes the others time out with an error instead of hanging.
# --------------------------------------------------------------------------
import ctypes
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    out = tmp_path_factory.mktemp("tp") / "libtp_harness.so"
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-pthread", "-I",
           str(HERE.parent / "minicpm-o-uya_b200" / "csrc"), "-o", str(out), str(HERE / "tp_protocol_harness.cpp")]
    subprocess.run(cmd, check=True, capture_output=True)
    lib = ctypes.CDLL(str(out))
    lib.tp_harness_run.restype = ctypes.c_int
    lib.tp_harness_run.argtypes = ([ctypes.c_int, ctypes.c_uint] + [ctypes.c_int] * 5 +
                                   [ctypes.c_ulonglong, ctypes.c_int, ctypes.c_uint, ctypes.POINTER(ctypes.c_int),
                                    ctypes.POINTER(ctypes.c_int)])
    return lib


def _run(lib, world, steps, nx=8, rows=96, kill_rank=-1, kill_step=0, limit_ms=300, skew_us=50, seed=1, first_step=1):
    status = (ctypes.c_int * world)()
    bad = (ctypes.c_int * world)()
    assert lib.tp_harness_run(world, first_step, steps, nx, rows, kill_rank, kill_step, limit_ms * 1_000_000, skew_us,
                              seed, status, bad) == 1
    return list(status), list(bad)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_protocol_sums_in_rank_order(harness, world):
    status, bad = _run(harness, world, steps=40, skew_us=30, seed=world)
    assert status == [0] * world and bad == [0] * world


def test_exchange_protocol_tags_wrap(harness):
    """The 32-bit exchange index wraps without a reset: steps whose indices
    cross 2^32 still tag every value apart from the slot's previous
    exchange and from the zeroed buffer."""
    nx, rows = 8, 96
    first = (1 << 32) // nx - 5  # the index wraps a few steps in
    status, bad = _run(harness, 4, steps=12, nx=nx, rows=rows, first_step=first)
    assert status == [0] * 4 and bad == [0] * 4


@pytest.mark.parametrize("world,kill_rank,kill_step", [(2, 1, 3), (4, 2, 5), (8, 0, 2)])
def test_killed_rank_makes_the_others_time_out(harness, world, kill_rank, kill_step):
    import time

    t0 = time.perf_counter()
    status, bad = _run(harness, world, steps=10, kill_rank=kill_rank, kill_step=kill_step, limit_ms=200)
    elapsed = time.perf_counter() - t0
    assert status[kill_rank] == 2
    assert all(s == 1 for r, s in enumerate(status) if r != kill_rank), status  # timed out with an error
    assert bad == [0] * world  # every exchange before the kill summed correctly
    assert elapsed < 5.0
