"""CPU: the multi-GPU host logic of bench.py on 2 gloo ranks (127.0.0.1):
max-over-ranks timing, barriers and the whole-job throughput formula."""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "foundation-pose-inference-library_b200" / "python"))
    from fp_b200.dist_utils import barrier, max_over_ranks, sum_over_ranks, world as w

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        assert w() == (rank, world)
        barrier()
        ms = 10.0 + 5.0 * rank  # rank 1 is the slower one
        m = max_over_ranks(ms)
        total_hyp = sum_over_ranks(252.0)
        q.put((rank, m, total_hyp, total_hyp / (m / 1000.0)))
        barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_timing_rules():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, m, total, value in res:
        assert m == 15.0  # max over ranks, on every rank
        assert total == 504.0
        assert abs(value - 504.0 / 0.015) < 1e-6
