"""GPU test of wp_gemm_q_noalloc, the GEMM + per-row re-quantisation entry point that allocates
no device memory.  It is meant for callers that cannot call cudaMalloc when they run it: a
process whose framework already handed the GPU's memory to its own caching allocator, or a
latency-bound thread that must not block in cudaMalloc.  Instead of growing a staging buffer
like wp_gemm_q, it stages through one fixed array inside the library.

The test calls it through the C ABI and compares it with wp_gemm_q (the existing entry point)
bit for bit, the tolerance every GEMM test here uses, on two calls in a row.  The second call
has fewer rows and much smaller values, so leftover per-row maxima from the first call would
show up as wrong scales.  It also checks that oversized calls are rejected.  This file sorts
last so that a run that stops at the first failure has already run every other test.  It
builds its own context and buffers, so it passes alone in a fresh process as well.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ctx(L, w):
    ctx = L.wp_create(w.ctypes.data, w.nbytes)
    assert ctx, "wp_create failed"
    return ctx


def _run(L, ctx, fn, q, s, t, k, n, ws, bias_p, dev):
    pq, ps = dev.put(q), dev.put(s)
    oq, osc = dev.empty(t * n), dev.empty(t * 4)
    assert fn(ctx, pq, ps, t, k, 0, n, ws, bias_p, None, oq, osc) == 0
    assert L.wp_sync(ctx) == 0
    return dev.get(oq, (t, n), np.int8), dev.get(osc, (t,), np.float32)


def test_noalloc_gemm_q_matches_gemm_q_twice(gpu_lib, dev):
    L = gpu_lib
    k, n = 512, 2048
    rng = np.random.default_rng(123)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    b = (0.3 * rng.standard_normal(n)).astype(np.float32)
    ctx = _ctx(L, w)
    try:
        pb = dev.put(b)
        ws = 1.0 / (73.6 * np.sqrt(k))
        for call, (t, scale) in enumerate([(400, 30.0), (137, 0.01)]):
            q = rng.integers(-127, 128, size=(t, k), dtype=np.int8)
            s = (scale * rng.uniform(0.5, 1.5, size=t)).astype(np.float32)
            ref_q, ref_s = _run(L, ctx, L.wp_gemm_q, q, s, t, k, n, ws, pb, dev)
            got_q, got_s = _run(L, ctx, L.wp_gemm_q_noalloc, q, s, t, k, n, ws, pb, dev)
            np.testing.assert_array_equal(got_s, ref_s, err_msg=f"call {call}")
            np.testing.assert_array_equal(got_q, ref_q, err_msg=f"call {call}")
    finally:
        L.wp_destroy(ctx)


def test_noalloc_rejects_oversized_calls(gpu_lib, dev):
    L = gpu_lib
    k, n = 64, 2048
    w = np.ones((n, k), np.int8)
    ctx = _ctx(L, w)
    try:
        t = 1024                                   # t * n = 2 Mi elements > 1 Mi limit
        pq, ps = dev.empty(t * k), dev.empty(t * 4)
        oq, osc = dev.empty(t * n), dev.empty(t * 4)
        assert L.wp_gemm_q_noalloc(ctx, pq, ps, t, k, 0, n, 1.0, None, None, oq, osc) == -22
        assert L.wp_gemm_q_noalloc(ctx, pq, ps, 0, k, 0, n, 1.0, None, None, oq, osc) == 0
        assert L.wp_gemm_q_noalloc(ctx, None, ps, 4, k, 0, n, 1.0, None, None, oq, osc) == -1
        assert L.wp_sync(ctx) == 0
    finally:
        L.wp_destroy(ctx)
