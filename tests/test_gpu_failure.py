"""Failure detection on the GPU without a GPU fault: bounded waits that are
made to run out, and the engine's abort path.

- q4k_tp_sum_parts, the receiving half of the fused tensor-parallel sum,
  reads tagged partial sums with the same bounded device wait the decode
  step uses. With every tag right it must equal residual + the ranks' sum in
  rank order (bit for bit); with one rank's words left at an old tag (a
  peer that never wrote this step) the wait must give up after its short
  limit, the call must report Q4K_ETIMEOUT, and the context must stay usable
  (a following call succeeds).
- An aborted engine fails every later call with Q4K_ETIMEOUT, and
  set_limits rejects a negative host limit.
"""
import time

import numpy as np
import pytest

import q4kb200 as q

pytestmark = pytest.mark.gpu

WORLD, COUNT = 3, 2560


def _words(values: np.ndarray, tags: np.ndarray) -> np.ndarray:
    return (tags.astype(np.uint64) << np.uint64(32)) | values.astype(np.float32).view(np.uint32).astype(np.uint64)


def _call(cuda, parts, residual, tag, wait_ns):
    L = q.lib()
    d_parts = cuda.from_numpy(parts.view(np.int64)).cuda()
    d_res = cuda.from_numpy(residual).cuda()
    out = cuda.full((COUNT,), float("nan"), device="cuda")
    err = cuda.zeros(4, dtype=cuda.int32, device="cuda")
    t0 = time.monotonic()
    st = L.q4k_tp_sum_parts(d_parts.data_ptr(), WORLD, COUNT, tag, d_res.data_ptr(), out.data_ptr(), wait_ns,
                            err.data_ptr(), None)
    return st, time.monotonic() - t0, out.cpu().numpy()


def test_tagged_sum_in_rank_order_then_a_stale_rank_times_out(cuda):
    rng = np.random.default_rng(5)
    vals = rng.standard_normal((WORLD, COUNT)).astype(np.float32)
    residual = rng.standard_normal(COUNT).astype(np.float32)
    tag = 41
    good = _words(vals, np.full((WORLD, COUNT), tag, np.uint32))
    st, _, out = _call(cuda, good, residual, tag, 2_000_000_000)
    q.check(st)
    want = vals[0].copy()
    for r in range(1, WORLD):
        want = (want + vals[r]).astype(np.float32)
    want = (residual + want).astype(np.float32)
    assert np.array_equal(out, want)

    # rank 2 never wrote the second half of this step: its words keep the previous tag
    stale_tags = np.full((WORLD, COUNT), tag, np.uint32)
    stale_tags[2, COUNT // 2:] = tag - 1
    stale = _words(vals, stale_tags)
    st, elapsed, _ = _call(cuda, stale, residual, tag, 5_000_000)  # 5 ms limit
    assert st == q.ETIMEOUT, (st, q.lib().q4k_last_error())
    assert elapsed < 2.0, elapsed

    # the context is still usable and the next step is exact again
    st, _, out = _call(cuda, good, residual, tag, 2_000_000_000)
    q.check(st)
    assert np.array_equal(out, want)


def test_aborted_engine_refuses_further_steps(cuda):
    from tiny_model import TINY, engine_config, tiny_tensors

    eng = q.Engine(engine_config(TINY, capacity=8))
    try:
        for n, (t, a, b, d) in tiny_tensors().items():
            eng.set_tensor(n, t, a, b, d)
        with pytest.raises(q.InvalidArgument):
            eng.set_limits(0, -1)
        eng.set_limits(1_000_000_000, 5_000)
        first, _, _ = eng.decode(7, 0)
        eng.abort()
        with pytest.raises(q.Timeout):
            eng.decode(first, 1)
        with pytest.raises(q.Timeout):
            eng.prefill([1, 2, 3], 0)
    finally:
        eng.close()
