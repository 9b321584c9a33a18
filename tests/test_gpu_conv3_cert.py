"""conv3 fused with the certified row quantisation of its output (the engine's conv3 path).

y3 feeds only quant(y3, FLAT) (src/model.rs:489), so the kernel sums the conv3 products with fused
multiply-adds, bounds the difference to the reference's dotf order (src/kernels.rs:172-183,
src/model.rs:446-468), and evaluates the row maximum and every element near a rounding boundary
in the reference's order.  The int8 rows and scales must equal the oracle's quant(conv3(y2)) bit
for bit: on random windows, on several windows stacked into one call, and on windows of zeros,
of a single non-zero input, and of very large or very small magnitudes.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PREP = 576 * 192 + 192


def _y2(rng, t1, scale=1.0):
    y = np.maximum(rng.standard_normal((t1, 64, 41)), 0.0) * scale
    y[:, :, 40] = 0.0
    return y.astype(np.float32)


def _c3(rng):
    return (rng.standard_normal((192, 64, 3, 3)) * np.sqrt(2.0 / 576)).astype(np.float32)


def _run(L, dev, y2, c3, lens=None):
    rows = y2.shape[0]
    py2, pc3, pprep = dev.put(y2), dev.put(c3), dev.empty(PREP * 4)
    pq, ps = dev.empty(rows * 3840), dev.empty(rows * 4)
    if lens is None:
        assert L.wasr_conv3_quant(py2, pc3, pprep, None, 0, rows, pq, ps, None) == 0
    else:
        roff = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        assert L.wasr_conv3_quant(py2, pc3, pprep, dev.put(roff), len(lens), rows, pq, ps, None) == 0
    return dev.get(pq, (rows, 3840), np.int8), dev.get(ps, (rows,), np.float32)


def _want(orc, y2, c3, lens):
    qs, ss, r = [], [], 0
    for n in lens:
        q, s = orc.quant(orc.conv3(y2[r:r + n], c3))
        qs.append(q)
        ss.append(s)
        r += n
    return np.concatenate(qs), np.concatenate(ss)


@pytest.mark.parametrize("t1", [1, 3, 4, 5, 57, 400])
def test_conv3_cert_one_window(gpu_lib, dev, orc, t1):
    rng = np.random.default_rng(t1)
    y2, c3 = _y2(rng, t1), _c3(rng)
    q, s = _run(gpu_lib, dev, y2, c3)
    wq, ws = _want(orc, y2, c3, [t1])
    np.testing.assert_array_equal(s.view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(q, wq)


def test_conv3_cert_stacked_windows(gpu_lib, dev, orc):
    """Windows stacked into one call: no patch reaches across a window boundary."""
    rng = np.random.default_rng(11)
    lens = [5, 1, 13, 2, 7, 64, 3]
    y2, c3 = _y2(rng, sum(lens)), _c3(rng)
    q, s = _run(gpu_lib, dev, y2, c3, lens)
    wq, ws = _want(orc, y2, c3, lens)
    np.testing.assert_array_equal(s.view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(q, wq)


def test_conv3_cert_special_windows(gpu_lib, dev, orc):
    """A window of zeros (every element a candidate: the all-exact path), one non-zero input,
    and magnitudes near 1e-25 and 1e20."""
    rng = np.random.default_rng(12)
    c3 = _c3(rng)
    z = np.zeros((6, 64, 41), np.float32)
    one = np.zeros((5, 64, 41), np.float32)
    one[2, 17, 9] = 3.0
    tiny = _y2(rng, 9, 1e-25)
    huge = _y2(rng, 6, 1e20)
    mixed = _y2(rng, 8)
    mixed[3] = 0.0
    parts = [z, one, tiny, huge, mixed]
    lens = [p.shape[0] for p in parts]
    y2 = np.concatenate(parts)
    q, s = _run(gpu_lib, dev, y2, c3, lens)
    wq, ws = _want(orc, y2, c3, lens)
    np.testing.assert_array_equal(s.view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(q, wq)
