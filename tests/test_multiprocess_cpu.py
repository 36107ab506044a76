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


def test_shard_ranges_cover_hypotheses_in_order():
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "foundation-pose-inference-library_b200" / "python"))
    from fp_b200.sharded import shard_range

    for n in (1, 7, 42, 252):
        for world in (1, 2, 3, 4, 8):
            if world > n:
                continue
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0
            for (b0, c0), (b1, _) in zip(ranges, ranges[1:]):
                assert b0 + c0 == b1
            assert sum(c for _, c in ranges) == n
            assert max(c for _, c in ranges) - min(c for _, c in ranges) <= 1
    assert [shard_range(252, 8, r)[1] for r in range(8)] == [32] * 4 + [31] * 4
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _shard_worker(rank, world, port, n, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "foundation-pose-inference-library_b200" / "python"))
    from fp_b200.sharded import gather_shards, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        begin, count = shard_range(n, world, rank)
        per = -(-n // world)
        # Stand-in for fp_register_shard_begin: row i of the shard carries its
        # global hypothesis index; padding rows are poison.
        local = torch.full((per, 4), -1.0)
        local[:count] = torch.arange(begin, begin + count, dtype=torch.float32)[:, None]
        full = gather_shards(local, n)
        q.put((rank, full[:, 0].tolist(), (full[:, 1:] == full[:, :1]).all().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,world", [(42, 2), (11, 3)])
def test_gather_shards_assembles_hypothesis_order(n, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = [q.get(timeout=5) for _ in range(world)]
    for _, order, rows_ok in res:
        assert order == [float(i) for i in range(n)]  # every rank, same order, no padding
        assert rows_ok


def _failing_rank_worker(rank, world, port, q):
    """Rank 1 fails between steps (an exception before its shard's gather, as
    a failed fp_register_shard_begin would raise) and leaves; rank 0 must get
    an error from its gather within the process group's short timeout
    instead of waiting for good."""
    import sys
    import time
    from datetime import timedelta
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "foundation-pose-inference-library_b200" / "python"))
    from fp_b200.sharded import gather_shards

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    n = 8
    local = torch.zeros((-(-n // world), 4))
    gather_shards(local, n)  # one good step on every rank
    if rank == 1:
        q.put((rank, "raised"))
        raise SystemExit(3)  # the failing rank leaves without joining the next gather
    t0 = time.monotonic()
    try:
        gather_shards(local, n)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        q.put((rank, f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}"))


def test_failed_rank_ends_peer_gather_with_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode is not None for p in procs)  # nobody hangs
    assert procs[1].exitcode == 3
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[1] == "raised"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2]) < 60.0
