"""Distributed host logic on CPU (no GPU): the reference collective contracts
(projects/titan-distributed/tests/collective.rs:6-49) and world_size-2 gloo runs
of the sharded-GEMM gather path and of failure detection.
"""
import datetime
import multiprocessing as mp
import socket

import numpy as np
import pytest

from titan_rs_b200 import distributed as D


def test_local_ring_matches_reference_tests():
    assert D.LocalRing().all_reduce_sum([[1.0, 2.0], [3.0, 4.0]]) == [4.0, 6.0]
    assert D.LocalRing().reduce_scatter_sum([[1.0, 2.0, 3.0, 4.0], [1.0, 1.0, 1.0, 1.0]]) == [[2.0, 3.0], [4.0, 5.0]]
    assert D.LocalRing().all_gather([[1.0, 2.0], [3.0]]) == [1.0, 2.0, 3.0]
    with pytest.raises(D.CollectiveError) as e:
        D.LocalRing().all_gather([])
    assert e.value.kind == "EmptyWorld"
    with pytest.raises(D.CollectiveError) as e:
        D.LocalRing().all_reduce_sum([[1.0], [1.0, 2.0]])
    assert e.value.kind == "InconsistentLengths"


def test_local_transport_checks_run_epoch_sequence_timeout_and_checksum():
    t = datetime.timedelta(milliseconds=1)
    sender, receiver = D.LocalTransport("run-a", 7, t), D.LocalTransport("run-a", 7, t)
    frame = sender.send(b"payload", t)
    assert receiver.receive(frame, t) == b"payload"
    for other, kind in ((D.LocalTransport("run-b", 7, t), "RunMismatch"), (D.LocalTransport("run-a", 8, t),
                                                                            "EpochMismatch"),
                        (receiver, "SequenceMismatch")):
        with pytest.raises(D.CollectiveError) as e:
            other.receive(frame, t)
        assert e.value.kind == kind
    with pytest.raises(D.CollectiveError) as e:
        sender.send(b"x", datetime.timedelta(0))
    assert e.value.kind == "Timeout"
    corrupt = sender.send(b"payload", t)
    corrupt.checksum = "broken"
    verifier = D.LocalTransport("run-a", 7, t)
    verifier.receive(frame, t)
    with pytest.raises(D.CollectiveError) as e:
        verifier.receive(corrupt, t)
    assert e.value.kind == "ChecksumMismatch"
    assert D.checksum(b"") == "cbf29ce484222325"


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
