"""Distributed host logic on CPU (no GPU): the even shards and the re-layout of the
sharded GEMM's gather, and world_size-2 gloo runs of the gather path and of failure
detection (the Collective trait, projects/titan-distributed/src/lib.rs:95-99).
"""
import datetime
import multiprocessing as mp
import socket

import numpy as np
import pytest

from titan_rs_b200 import distributed as D


def test_even_shard_and_reassembly():
    assert D.even_shard(8192, 8, 3) == (3072, 4096)
    with pytest.raises(ValueError):
        D.even_shard(10, 4, 0)
    full = np.arange(6 * 8).reshape(6, 8)
    blocks = np.stack([full[:, r * 2:(r + 1) * 2] for r in range(4)])
    np.testing.assert_array_equal(D.reassemble_column_blocks(blocks, 4), full)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gemm_rank(rank, world, port, q):
    import torch.distributed as dist

    import oracle
    from titan_rs_b200 import distributed as Dd
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        rng = np.random.default_rng(0)  # every rank builds the same A and B
        m, n, k = 16, 24, 8
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (n, k)).astype(np.float32)  # column-major B stored [N, K]
        lo, hi = Dd.even_shard(n, world, rank)
        block = oracle.gemm(a, b[lo:hi], transpose_rhs=True)  # this rank's C[:, lo:hi]
        gathered = Dd.ProcessGroupCollective().all_gather([block.ravel()])
        c = Dd.reassemble_column_blocks(np.array(gathered, np.float32).reshape(world, m, hi - lo), world)
        q.put((rank, bool(np.array_equal(c, oracle.gemm(a, b, transpose_rhs=True)))))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))


def _failure_rank(rank, world, port, q):
    import torch.distributed as dist

    from titan_rs_b200 import distributed as Dd
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=3))
        if rank == 1:
            q.put((rank, "left"))
            return  # leaves between steps, without joining the next collective
        try:
            Dd.ProcessGroupCollective().all_gather([[1.0, 2.0]])
            q.put((rank, "completed"))
        except Exception as exc:
            q.put((rank, "error:" + type(exc).__name__))
    except Exception as exc:
        q.put((rank, "setup:" + repr(exc)))


def _run(target, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, value = q.get(timeout=timeout)
        results[rank] = value
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


def test_two_rank_sharded_gemm_gather_is_exact():
    results = _run(_gemm_rank)
    assert results == {0: True, 1: True}, results


def test_lost_rank_surfaces_as_an_error_not_a_hang():
    results = _run(_failure_rank)
    assert results[1] == "left"
    assert results[0].startswith("error:"), results


@pytest.mark.parametrize("units,world", [(256, 8), (256, 3), (6, 4), (2, 4), (64, 8), (1, 1)])
def test_shard_units_cover_every_unit_once(units, world):
    spans = [D.shard_units(units, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == units
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1
    if units % world == 0:
        assert spans == [D.even_shard(units, world, r) for r in range(world)]
    with pytest.raises(ValueError):
        D.shard_units(units, world, world)
