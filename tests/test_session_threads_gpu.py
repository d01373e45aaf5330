"""One tb_session driven from several host threads at once.

The reference's CUDA session is `Send + Sync`: its registries sit behind mutexes and
every call re-activates the context (projects/titan-backend-cuda/src/lib.rs:1170-1176,
1576), so any thread may allocate, upload, launch, wait and drop buffers on a shared
session. Here four Python threads share one Session (ctypes releases the GIL around
every library call, so the native entry points really do run concurrently). Each
thread, on its own stream:

- runs softmax (fp32) and a bf16 GEMM through the Runtime and checks them against the
  CPU oracle;
- uploads a buffer and hands the buffer and the upload's event to the next thread,
  which orders its own stream after that event (wait_event: a cross-stream edge, no
  host wait), copies the buffer, downloads the copy and checks the bytes; every other
  round it also polls and host-waits on the other thread's event;
- releases the other thread's buffer once its download has returned, while the other
  threads keep working.
"""
import math
import queue
import threading

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200.kernel_abi import DType

from gpu_util import elementwise_rel_err, max_rel_err

pytestmark = pytest.mark.gpu

THREADS = 4
ROUNDS = 12


def test_one_session_driven_from_four_host_threads():
    s = tb.Session(0)
    errors = []
    inbox = [queue.Queue() for _ in range(THREADS)]
    checked = [0] * THREADS
    start = threading.Barrier(THREADS)

    def worker(t):
        try:
            rt = tb.Runtime(s)  # its own stream
            rng = np.random.default_rng(100 + t)
            start.wait(timeout=60)
            for r in range(ROUNDS):
                x = (rng.standard_normal((64, 512)) * 2.0).astype(np.float32)
                hs = rt.execute(tb.OpRequest("softmax", [tb.TensorHandle.from_numpy(s, x, DType.F32, rt.stream)],
                                             [tb.TensorSpec(DType.F32, x.shape)]))
                m, n, k = 128 + 64 * (t % 2), 256, 64 * (1 + r % 3)
                a = tb.fill_normal(m * k, seed=1000 * t + r, dtype=DType.BF16).reshape(m, k)
                b = tb.fill_normal(n * k, seed=2000 * t + r, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape(n, k)
                hg = rt.execute(tb.OpRequest("gemm", [tb.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream),
                                                      tb.TensorHandle.from_numpy(s, b, DType.BF16, rt.stream)],
                                             [tb.TensorSpec(DType.BF16, (m, n))], {"transpose_rhs": True}))

                payload = rng.integers(0, 256, 4096 + 64 * t, dtype=np.uint8)
                buf = s.allocate(payload.nbytes)
                ev = s.upload(rt.stream, buf, payload)
                inbox[(t + 1) % THREADS].put((ev, buf, payload))
                del ev, buf  # the receiving thread owns them now

                ev2, buf2, expected = inbox[t].get(timeout=120)
                if r % 2:
                    s.poll(ev2)  # either answer is fine; it must not fail or race
                    s.wait(ev2)  # host wait on another thread's event
                s.wait_event(rt.stream, ev2)  # this stream now runs after the other thread's upload
                dst = s.allocate(expected.nbytes)
                s.copy(rt.stream, dst, buf2, expected.nbytes)
                got = np.empty_like(expected)
                s.download(rt.stream, dst, got)  # finishes before it returns
                assert np.array_equal(got, expected), f"thread {t} round {r}: cross-thread copy differs"
                buf2.release()  # the other thread's buffer, dropped here while the others keep running
                dst.release()

                hs.wait()
                err = elementwise_rel_err(hs.outputs[0].to_numpy(rt.stream), oracle.softmax(x))
                assert err <= 1e-5, f"thread {t} round {r}: softmax rel err {err}"
                hg.wait()
                ref = oracle.gemm_bf16_points(a, b, True, m, n, k, np.repeat(np.arange(m), n),
                                              np.tile(np.arange(n), m)).reshape(m, n)
                err = max_rel_err(hg.outputs[0].to_f32(rt.stream), ref)
                assert err <= 1e-2, f"thread {t} round {r}: gemm err {err}"
                checked[t] += 1
        except Exception as e:  # reported by the main thread
            errors.append((t, repr(e)))

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(THREADS)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads), "a worker thread did not finish"
    assert not errors, errors
    assert checked == [ROUNDS] * THREADS
    s.close()
