"""The engine's fused feed-forward up-projection: f1 GEMM + GELU + per-row int8 quantisation in
one tcgen05 kernel (src/model.rs:495-496, then quant of src/kernels.rs:11-25), through the
wasr_gemm_gelu_quant parity hook.

The kernel never stores the fp32 f1 output: it takes each row's exact max x in a first pass over
the MMAs, quantises the certified GELU approximation in a second, and re-evaluates the exact GELU
where a rounding test cannot decide.  Rows it cannot certify (a non-finite x, or a maximum that
may lie on the negative side of the GELU) go to an exact kernel.  The int8 rows and scales must
equal the oracle's quant(gelu(qgemm(...))) bit for bit: on random shapes, on rows built for the
exact kernel, on rows near the certified path's limits, and with per-channel or per-tensor
weight scales.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(L, dev, a, xs, w, ws, ws_vec, bias):
    m, k = a.shape
    n = w.shape[0]
    pq, ps = dev.empty(max(m * n, 1)), dev.empty(max(m * 4, 4))
    work = dev.put(np.zeros(m + 2, np.int32))
    rc = L.wasr_gemm_gelu_quant(dev.put(a), dev.put(xs), dev.put(w), float(ws),
                                None if ws_vec is None else dev.put(ws_vec),
                                None if bias is None else dev.put(bias), m, k, n, pq, ps, work, None)
    assert rc == 0
    wk = dev.get(work, (m + 2,), np.int32)
    assert wk[0] == 0, f"device error word {wk[0]}"
    return dev.get(pq, (m, n), np.int8), dev.get(ps, (m,), np.float32), int(wk[1])


def _want(orc, a, xs, w, ws, ws_vec, bias):
    x = orc.qgemm(a, xs, w, ws, ws_vec, bias)
    return orc.quant(orc.gelu(x))


def _case(rng, m, k, n, per_channel=True, with_bias=True):
    a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    xs = rng.uniform(0.002, 0.02, m).astype(np.float32)
    ws_vec = rng.uniform(0.5, 1.5, n).astype(np.float32) / np.float32(127 * np.sqrt(k)) if per_channel else None
    ws = np.float32(1.0 / (127 * np.sqrt(k)))
    bias = (0.1 * rng.standard_normal(n)).astype(np.float32) if with_bias else None
    return a, xs, w, ws, ws_vec, bias


def _exact_rows(orc, args):
    """Rows the kernel must leave to the exact kernel: some x non-finite, or gelu(max x) < 0.171."""
    x = orc.qgemm(*args)
    fin = np.isfinite(x).all(axis=1)
    mx = np.where(fin, np.max(np.where(fin[:, None], x, 0.0), axis=1), 0.0).astype(np.float32)
    return int(np.sum(~fin | ~(orc.gelu(mx) >= np.float32(0.171))))


def _check(L, dev, orc, args):
    q, s, nfix = _run(L, dev, *args)
    wq, ws_ = _want(orc, *args)
    np.testing.assert_array_equal(s.view(np.uint32), ws_.view(np.uint32))
    np.testing.assert_array_equal(q, wq)
    assert nfix == _exact_rows(orc, args)
    return nfix


# 9729 rows: 77 row blocks of 128, more than half of the 148 SMs
@pytest.mark.parametrize("m,k,n", [(1, 512, 2048), (127, 512, 2048), (300, 512, 2048), (4097, 512, 2048),
                                   (9729, 512, 2048), (200, 128, 256), (333, 1024, 1024)])
def test_gemm_gelu_q_random(gpu_lib, dev, orc, m, k, n):
    rng = np.random.default_rng(m * 7 + k + n)
    assert _check(gpu_lib, dev, orc, _case(rng, m, k, n)) == 0


def test_gemm_gelu_q_per_tensor_scale_no_bias(gpu_lib, dev, orc):
    rng = np.random.default_rng(5)
    assert _check(gpu_lib, dev, orc, _case(rng, 515, 512, 2048, per_channel=False, with_bias=False)) == 0


def test_gemm_gelu_q_exact_rows(gpu_lib, dev, orc):
    """Rows the certified path leaves to the exact kernel: a NaN or infinite row scale (non-finite
    x), rows whose every x is negative (the largest |gelu| may lie below 0), rows whose max x sits
    just below or above the point where gelu reaches 0.171; and, between them, ordinary rows, rows
    of a zero scale (x = bias) and rows of huge x."""
    rng = np.random.default_rng(6)
    a, xs, w, ws, ws_vec, bias = _case(rng, 260, 512, 2048)
    bias = bias.copy()
    xs = xs.copy()
    xs[3] = np.nan
    xs[70] = np.inf
    xs[71] = -np.inf
    xs[130] = 0.0                  # x = bias everywhere
    xs[131] = 1e30                 # huge x: gelu(x) = x, scale near 1e36
    for r in (10, 11, 200):        # every x negative: x = bias < 0
        xs[r] = 0.0
    bias_neg = -np.abs(bias) - 0.5
    a2, xs2 = a.copy(), xs.copy()
    # rows 10, 11, 200 use a second call with all-negative biases (a row's bias is shared by all
    # rows, so the negative-bias rows are checked in a call of their own)
    assert _check(gpu_lib, dev, orc, (a, xs, w, ws, ws_vec, bias)) >= 3  # the NaN, the infinite scales
    assert _check(gpu_lib, dev, orc, (a2, xs2, w, ws, ws_vec, bias_neg)) >= 3 + 4  # and x = bias < 0
    # max x near the threshold: scale rows so that their largest x is 0.25 .. 0.40
    x = orc.qgemm(a, np.ones_like(xs), w, ws, ws_vec, None)
    xs3 = (np.linspace(0.25, 0.40, a.shape[0]) / np.max(x, axis=1)).astype(np.float32)
    n3 = _check(gpu_lib, dev, orc, (a, xs3, w, ws, ws_vec, None))
    assert 0 < n3 < a.shape[0]


def test_gemm_gelu_q_near_tied_and_boundary_rows(gpu_lib, dev, orc):
    """Weight rows repeated so that several columns of a row share the exact maximum, and large
    activations, so that many scaled values land close to rounding boundaries."""
    rng = np.random.default_rng(7)
    a, xs, w, ws, ws_vec, bias = _case(rng, 400, 512, 2048)
    w = w.copy()
    w[1000:1010] = w[5]
    ws_vec = ws_vec.copy()
    ws_vec[1000:1010] = ws_vec[5]
    bias = bias.copy()
    bias[1000:1010] = bias[5]
    assert _check(gpu_lib, dev, orc, (a, xs * np.float32(8.0), w, ws, ws_vec, bias)) == 0


def test_gemm_gelu_q_bounded_wait_runs_out_and_recovers(gpu_lib, dev, orc):
    """The producer issues no loads, so the MMA warp's bounded wait (1 ms) runs out with nothing
    in flight: the kernel records an error code and returns (no fault, no hang), and the next
    call on the same stream is bit-exact again."""
    L = gpu_lib
    rng = np.random.default_rng(12)
    a, xs, w, ws, ws_vec, bias = _case(rng, 300, 512, 2048)
    m, n = a.shape[0], w.shape[0]
    pa, px, pw, pv, pb = dev.put(a), dev.put(xs), dev.put(w), dev.put(ws_vec), dev.put(bias)
    pq, ps = dev.empty(m * n), dev.empty(m * 4)
    work = dev.put(np.zeros(m + 2, np.int32))
    assert L.wasr_gemm_gelu_quant_wait_probe(pa, px, pw, float(ws), pv, pb, m, 512, n, pq, ps, work,
                                             1_000_000, None) == 0
    wk = dev.get(work, (m + 2,), np.int32)
    assert wk[0] in (1, 2, 3), f"error word {wk[0]}"
    assert wk[1] == 0
    _check(L, dev, orc, (a, xs, w, ws, ws_vec, bias))


def test_gemm_gelu_q_twice_same_result(gpu_lib, dev, orc):
    """Two calls in a row on the same buffers: the row list is reset per call."""
    rng = np.random.default_rng(8)
    args = _case(rng, 333, 512, 2048)
    xs = args[1].copy()
    xs[7] = np.nan
    args = (args[0], xs) + args[2:]
    q1, s1, n1 = _run(gpu_lib, dev, *args)
    q2, s2, n2 = _run(gpu_lib, dev, *args)
    assert n1 == n2 == 1
    np.testing.assert_array_equal(q1, q2)
    np.testing.assert_array_equal(s1.view(np.uint32), s2.view(np.uint32))
