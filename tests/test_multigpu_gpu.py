"""Multi-GPU path: NCCL all-gather (Collective::all_gather on device buffers), the
N-sharded GEMM, and attention / conv2d sharded over batch x heads / batch. The
one-rank cases run on any single B200; the two-rank cases run as child processes
when at least two GPUs are visible (NVLS off, as this pool requires for
multi-process GPU tests). Sharded results are compared with the unsharded kernel
of the same family bit for bit and with the CPU oracle on sampled points."""
import math
import multiprocessing as mp
import os

import numpy as np
import pytest

import titan_rs_b200 as tb
from titan_rs_b200 import distributed as D
from titan_rs_b200.kernel_abi import DType

pytestmark = pytest.mark.gpu


def _gemm_inputs(m, n, k, seed=21):
    a = tb.fill_normal(m * k, seed=seed * 16, dtype=DType.BF16).reshape(m, k)
    b = tb.fill_normal(n * k, seed=seed * 16 + 1, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape(n, k)
    return a, b


def _reference_c(s, rt, a, b, candidate="gemm_bf16_tn"):
    m, k = a.shape
    n = b.shape[0]
    ta = tb.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
    tbb = tb.TensorHandle.from_numpy(s, b, DType.BF16, rt.stream)
    # The sharded path runs a whole-K kernel on each shard; compare with the same kernel family.
    h = rt.execute(tb.OpRequest("gemm", [ta, tbb], [tb.TensorSpec(DType.BF16, (m, n))],
                                {"transpose_rhs": True, "candidate": candidate}))
    h.wait()
    return h.outputs[0].to_numpy()


def test_one_rank_sharded_gemm_equals_single_gpu_gemm():
    s = tb.Session(0)
    rt = tb.Runtime(s)
    m, n, k = 512, 768, 1024
    a, b = _gemm_inputs(m, n, k)
    ref = _reference_c(s, rt, a, b)
    coll = D.NcclCollective(s, D.new_comm_id(), 1, 0, timeout_ms=20000)
    ta = tb.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
    tbb = tb.TensorHandle.from_numpy(s, b, DType.BF16, rt.stream)
    c = tb.TensorHandle.allocate(s, DType.BF16, (m, n))
    ws = s.allocate(m * n * 2)
    coll.sharded_gemm(rt.stream, ta, tbb, c, ws)
    s.synchronize(rt.stream)
    np.testing.assert_array_equal(c.to_numpy(), ref)
    # all_gather with one rank is a copy.
    src = s.allocate(4096)
    dst = s.allocate(4096)
    s.wait(s.upload(rt.stream, src, np.arange(1024, dtype=np.float32)))
    coll.all_gather(rt.stream, src, dst, 4096)
    out = np.empty(1024, np.float32)
    s.download(rt.stream, dst, out)
    np.testing.assert_array_equal(out, np.arange(1024, dtype=np.float32))
    coll.close()
    s.close()


# (m, n, k, fused kernel, plain kernel of the same family): 25 output tiles of 128x256
# take the 1-SM kernel; 323 (with M and N tails) take CTA pairs.
FUSED_CASES = [(640, 1280, 1536, "gemm_bf16_tn_allgather", "gemm_bf16_tn"),
               (2056, 4856, 1024, "gemm_bf16_tn_allgather_2sm", "gemm_bf16_tn_2sm")]


@pytest.mark.parametrize("m,n,k,fused,plain", FUSED_CASES)
def test_one_rank_fused_sharded_gemm_equals_single_gpu_gemm(m, n, k, fused, plain):
    """A registered output takes the fused kernel; with one rank it must equal the plain
    whole-K GEMM of the same pipeline bit for bit, call after call."""
    s = tb.Session(0)
    rt = tb.Runtime(s)
    a, b = _gemm_inputs(m, n, k, seed=23)
    ref = _reference_c(s, rt, a, b, plain)
    coll = D.NcclCollective(s, D.new_comm_id(), 1, 0, timeout_ms=20000)
    ta = tb.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
    tbb = tb.TensorHandle.from_numpy(s, b, DType.BF16, rt.stream)
    c = tb.TensorHandle.allocate(s, DType.BF16, (m, n))
    coll.register_buffer(rt.stream, c.buffer)
    with pytest.raises(tb.HalError, match="already registered"):
        coll.register_buffer(rt.stream, c.buffer)
    for _ in range(2):
        coll.sharded_gemm(rt.stream, ta, tbb, c, None)
        s.synchronize(rt.stream)
        assert tb.last_candidate() == fused
        np.testing.assert_array_equal(c.to_numpy(), ref)
    coll.deregister_buffer(c.buffer)
    with pytest.raises(tb.HalError, match="not registered"):
        coll.deregister_buffer(c.buffer)
    coll.close()
    s.close()


def _oracle_ok(a, b, c_bits, samples=2048, seed=0):
    """Sampled points of C = A B^T (B stored [N, K]) against the CPU oracle."""
    import oracle
    m, k = a.shape
    n = b.shape[0]
    rng = np.random.default_rng(seed)
    rows = np.concatenate([rng.integers(0, m, samples), [0, m - 1, 0, m - 1]])
    cols = np.concatenate([rng.integers(0, n, samples), [0, 0, n - 1, n - 1]])
    ref = oracle.gemm_bf16_points(a, b, True, m, n, k, rows, cols)
    got = tb.bf16_bits_to_f32(c_bits[rows, cols])
    return bool(np.isfinite(got).all() and np.max(np.abs(got - ref)) <= 1e-2 * np.max(np.abs(ref)))


def _device_count() -> int:
    try:
        return len(tb.enumerate_devices())
    except Exception:
        return 0


def _rank_main(rank, world, q_in, q_out, mode):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import titan_rs_b200 as tbm
        from titan_rs_b200 import distributed as Dm
        s = tbm.Session(rank)
        rt = tbm.Runtime(s)
        if rank == 0:
            cid = Dm.new_comm_id()
            for _ in range(world - 1):
                q_in.put(cid)
        else:
            cid = q_in.get(timeout=60)
        coll = Dm.NcclCollective(s, cid, world, rank, timeout_ms=20000)
        if mode == "gemm":
            m, n, k = 384, 1024, 2048
            a, b = _gemm_inputs(m, n, k)
            ref = _reference_c(s, rt, a, b)
            lo, hi = Dm.even_shard(n, world, rank)
            ta = tbm.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
            tbs = tbm.TensorHandle.from_numpy(s, np.ascontiguousarray(b[lo:hi]), DType.BF16, rt.stream)
            c = tbm.TensorHandle.allocate(s, DType.BF16, (m, n))
            ws = s.allocate(m * n * 2)
            coll.sharded_gemm(rt.stream, ta, tbs, c, ws)
            s.synchronize(rt.stream)
            got = c.to_numpy()
            ok_gemm = bool(np.array_equal(got, ref)) and _oracle_ok(a, b, got)
            src, dst = s.allocate(1024 * 4), s.allocate(1024 * 4 * world)
            s.wait(s.upload(rt.stream, src, np.full(1024, rank, np.float32)))
            coll.all_gather(rt.stream, src, dst, 1024 * 4)
            out = np.empty(1024 * world, np.float32)
            s.download(rt.stream, dst, out)
            ok_gather = bool(np.array_equal(out, np.repeat(np.arange(world, dtype=np.float32), 1024)))
            coll.barrier(rt.stream)
            s.synchronize(rt.stream)
            q_out.put((rank, ok_gemm and ok_gather))
        elif mode in ("gemm_p2p", "gemm_p2p_pairs", "gemm_p2p_pushers"):
            # Fused GEMM + all-gather into registered outputs, twice with different inputs.
            if mode == "gemm_p2p":
                m, n, k = 520, 1536, 1024  # M is not a multiple of the 128-row tile
                fused, plain = "gemm_bf16_tn_allgather", "gemm_bf16_tn"
            elif mode == "gemm_p2p_pairs":
                m, n, k = 2056, 9712, 1024  # 323 tiles per shard, M and N tails: CTA pairs
                fused, plain = "gemm_bf16_tn_allgather_2sm", "gemm_bf16_tn_2sm"
            else:
                # Dedicated pusher CTAs (the default from 4 ranks), forced here for 2.
                os.environ["TITAN_B200_ALLGATHER_PUSHERS"] = "16"
                m, n, k = 2056, 9712, 1024
                fused, plain = "gemm_bf16_tn_allgather_2sm_push", "gemm_bf16_tn_2sm"
            lo, hi = Dm.even_shard(n, world, rank)
            c = tbm.TensorHandle.allocate(s, DType.BF16, (m, n))
            coll.register_buffer(rt.stream, c.buffer)
            ok = True
            for seed in (31, 32):
                a, b = _gemm_inputs(m, n, k, seed=seed)
                ref = _reference_c(s, rt, a, b, plain)
                ta = tbm.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
                tbs = tbm.TensorHandle.from_numpy(s, np.ascontiguousarray(b[lo:hi]), DType.BF16, rt.stream)
                coll.sharded_gemm(rt.stream, ta, tbs, c, None)
                s.synchronize(rt.stream)
                ok = ok and tbm.last_candidate() == fused
                got = c.to_numpy()
                ok = ok and bool(np.array_equal(got, ref)) and _oracle_ok(a, b, got, seed=seed)
            coll.barrier(rt.stream)
            s.synchronize(rt.stream)
            coll.deregister_buffer(c.buffer)
            q_out.put((rank, ok))
        elif mode == "gemm_c3":
            # C3 itself: 8192^3, B column-major N-sharded over the ranks, fused all-gather
            # into registered outputs; checked against the oracle on sampled points and by
            # the column-checksum identity 1^T C = (1^T A) B over every column.
            m = n = k = 8192
            a = tbm.fill_normal(m * k, seed=32, dtype=DType.BF16).reshape(m, k)
            b = tbm.fill_normal(n * k, seed=33, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape(n, k)
            lo, hi = Dm.even_shard(n, world, rank)
            c = tbm.TensorHandle.allocate(s, DType.BF16, (m, n))
            coll.register_buffer(rt.stream, c.buffer)
            ta = tbm.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
            tbs = tbm.TensorHandle.from_numpy(s, np.ascontiguousarray(b[lo:hi]), DType.BF16, rt.stream)
            coll.sharded_gemm(rt.stream, ta, tbs, c, None)
            s.synchronize(rt.stream)
            got = c.to_numpy()
            ok = tbm.last_candidate().startswith("gemm_bf16_tn_allgather") and _oracle_ok(a, b, got, 4096, rank)
            af = tbm.bf16_bits_to_f32(a).astype(np.float64)
            colsum_ref = af.sum(axis=0) @ tbm.bf16_bits_to_f32(b).astype(np.float64).T
            colsum = tbm.bf16_bits_to_f32(got).astype(np.float64).sum(axis=0)
            ok = ok and bool(np.max(np.abs(colsum - colsum_ref)) <= 1e-2 * np.max(np.abs(colsum_ref)))
            coll.barrier(rt.stream)
            s.synchronize(rt.stream)
            coll.deregister_buffer(c.buffer)
            q_out.put((rank, ok))
        elif mode in ("sdpa_shard", "conv_shard"):
            # No communication: every rank holds the whole seeded inputs, runs only its
            # units and checks them against the oracle.
            import oracle
            if mode == "sdpa_shard":
                bb, hh, t, d = 2, 4, 512, 128
                q, k, v = (tbm.fill_normal(bb * hh * t * d, seed=340 + i, dtype=DType.BF16).reshape(bb, hh, t, d)
                           for i in range(3))
                ins = [tbm.TensorHandle.from_numpy(s, x, DType.BF16, rt.stream) for x in (q, k, v)]
                req = tbm.OpRequest("scaled_dot_product_attention", ins, [tbm.TensorSpec(DType.BF16, q.shape)],
                                    {"causal": True})
                hdl, (lo, hi) = Dm.execute_local(rt, req, world, rank)
                hdl.wait()
                got = hdl.outputs[0].to_f32().reshape(-1, d)
                ref = oracle.sdpa_bf16_rows(q, k, v, bb, hh, t, t, d, True, np.arange(lo * t, hi * t))
            else:
                n, hw, cin, cout = 6, 28, 64, 256
                x = tbm.fill_normal(n * hw * hw * cin, seed=350, dtype=DType.BF16).reshape(n, hw, hw, cin)
                w = tbm.fill_normal(cout * 9 * cin, seed=351, std=math.sqrt(2.0 / (9 * cin)),
                                    dtype=DType.BF16).reshape(cout, 3, 3, cin)
                attrs = {"stride_h": 1, "stride_w": 1, "pad_h": 1, "pad_w": 1, "dilation_h": 1, "dilation_w": 1,
                         "groups": 1, "layout": "NHWC"}
                ins = [tbm.TensorHandle.from_numpy(s, x, DType.BF16, rt.stream),
                       tbm.TensorHandle.from_numpy(s, w, DType.BF16, rt.stream)]
                req = tbm.OpRequest("conv2d", ins, [tbm.TensorSpec(DType.BF16, (n, hw, hw, cout))], attrs)
                hdl, (lo, hi) = Dm.execute_local(rt, req, world, rank)
                hdl.wait()
                got = hdl.outputs[0].to_f32().ravel()
                per = hw * hw * cout
                ref = oracle.conv2d_nhwc_bf16_points(x, w, None, n, hw, hw, cin, cout, 3, 3, (1, 1), (1, 1), (1, 1),
                                                     hw, hw, np.arange(lo * per, hi * per))
            err = float(np.max(np.abs(got.ravel() - ref.ravel())) / np.max(np.abs(ref)))
            q_out.put((rank, (hi - lo > 0) and err <= 1e-2))
        elif mode in ("p2p_absent", "p2p_absent_pairs", "p2p_absent_pushers"):
            if mode == "p2p_absent_pushers":
                os.environ["TITAN_B200_ALLGATHER_PUSHERS"] = "16"
            # Rank 1 registers its output but never makes the call: rank 0's fused kernel
            # gives up its entry wait after ~1 s (a flag nothing sets), reports the code, and
            # its context stays usable. With CTA pairs the CTAs still run the pair pipeline
            # (stores off), so every cluster barrier is reached.
            m, n, k = (256, 512, 256) if mode == "p2p_absent" else (2056, 9712, 512)
            fused = {"p2p_absent": "gemm_bf16_tn_allgather", "p2p_absent_pairs": "gemm_bf16_tn_allgather_2sm",
                     "p2p_absent_pushers": "gemm_bf16_tn_allgather_2sm_push"}[mode]
            c = tbm.TensorHandle.allocate(s, DType.BF16, (m, n))
            coll.register_buffer(rt.stream, c.buffer)
            if rank == 0:
                a, b = _gemm_inputs(m, n, k, seed=33)
                lo, hi = Dm.even_shard(n, world, rank)
                ta = tbm.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
                tbs = tbm.TensorHandle.from_numpy(s, np.ascontiguousarray(b[lo:hi]), DType.BF16, rt.stream)
                coll.sharded_gemm(rt.stream, ta, tbs, c, None)
                try:
                    s.synchronize(rt.stream)
                    outcome = "no error"
                except tbm.HalError as e:
                    outcome = "timeout" if "47410501" in str(e) else repr(e)
                if tbm.last_candidate() != fused:
                    outcome = "ran " + tbm.last_candidate()
                # The context still runs work.
                probe = s.allocate(64)
                s.wait(s.upload(rt.stream, probe, np.arange(16, dtype=np.float32)))
                back = np.empty(16, np.float32)
                s.download(rt.stream, probe, back)
                usable = bool(np.array_equal(back, np.arange(16, dtype=np.float32)))
                q_in.put("done")
                q_out.put((rank, (outcome, usable)))
            else:
                q_in.get(timeout=120)
                q_out.put((rank, "absent"))
            coll.deregister_buffer(c.buffer)
        else:
            # Departure between steps: rank 1 announces it leaves and exits with nothing in flight;
            # rank 0 checks the announcement on the host before its next collective and stops.
            coll.barrier(rt.stream)
            s.synchronize(rt.stream)
            if rank == 1:
                q_in.put("departed")
                coll.close()
                q_out.put((rank, "left"))
                return
            msg = q_in.get(timeout=60)
            q_out.put((rank, "detected" if msg == "departed" else "missed"))
        coll.close()
        s.close()
    except Exception as exc:
        q_out.put((rank, repr(exc)))


def _spawn(world, mode):
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, q_in, q_out, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q_out.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_rank_sharded_gemm_and_all_gather():
    assert _spawn(2, "gemm") == {0: True, 1: True}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_rank_fused_sharded_gemm_over_peer_stores():
    assert _spawn(2, "gemm_p2p") == {0: True, 1: True}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_rank_fused_sharded_gemm_on_cta_pairs():
    assert _spawn(2, "gemm_p2p_pairs") == {0: True, 1: True}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_rank_fused_sharded_gemm_with_pusher_ctas():
    assert _spawn(2, "gemm_p2p_pushers") == {0: True, 1: True}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["p2p_absent", "p2p_absent_pairs", "p2p_absent_pushers"])
def test_two_rank_fused_gemm_gives_up_when_a_peer_never_arrives(mode):
    assert _spawn(2, mode) == {0: ("timeout", True), 1: "absent"}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_rank_fused_sharded_gemm_at_c3_against_the_oracle():
    assert _spawn(2, "gemm_c3") == {0: True, 1: True}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["sdpa_shard", "conv_shard"])
def test_two_rank_communication_free_shards_against_the_oracle(mode):
    assert _spawn(2, mode) == {0: True, 1: True}


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_rank_departure_is_detected_on_the_host():
    assert _spawn(2, "depart") == {0: "detected", 1: "left"}
