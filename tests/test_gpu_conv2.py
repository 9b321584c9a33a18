"""conv1 and conv2 of the conv frontend (src/model.rs:398-444) through the wasr_conv1 /
wasr_conv2 parity hooks.

conv1: the engine's kernel takes its 32 x 25 weights by value (a kernel argument), the reference
ABI's reads them from device memory; both must give the oracle's y1 bit for bit.

Two kernels compute it: the engine's position-pair kernel (c2t given: packed products
fma.rn(x, w, -0) and packed rounded adds per dotf lane) and the reference ABI's lane-pair kernel
(c2t NULL, behind wk_front).  Both keep the dotf order of src/kernels.rs:172-183, so y2 must equal
the oracle's bit for bit: on single windows of every length class, on ragged windows stacked into
one call (no patch may reach across a window), and on inputs with negative values and signed
zeros, with products that are subnormal, and with products that overflow.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

C2T = 64 * 1568


def _c2(rng, scale=0.03):
    return (rng.standard_normal((64, 32, 7, 7)) * scale).astype(np.float32)


def _y1(rng, t, scale=1.0):
    return (np.maximum(rng.standard_normal((t, 32, 40)), 0.0) * scale).astype(np.float32)


def _rows(t):
    return (t - 5) // 5 + 1 if t >= 5 else 0


def _run(L, dev, y1, c2, lens, engine):
    frames = y1.shape[0]
    rows = sum(_rows(t) for t in lens)
    py1, pc2 = dev.put(y1), dev.put(c2)
    pc2t = dev.empty(C2T * 4) if engine else None
    py2 = dev.put(np.full((rows, 64, 41), np.nan, np.float32))
    if len(lens) == 1:
        rc = L.wasr_conv2(py1, pc2, pc2t, None, None, 0, frames, rows, py2, None)
    else:
        foff = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        roff = np.concatenate([[0], np.cumsum([_rows(t) for t in lens])]).astype(np.int32)
        rc = L.wasr_conv2(py1, pc2, pc2t, dev.put(foff), dev.put(roff), len(lens), frames, rows, py2, None)
    assert rc == 0
    return dev.get(py2, (rows, 64, 41), np.float32)


def _want(orc, y1, c2, lens):
    out, f = [], 0
    for t in lens:
        out.append(orc.conv2(y1[f:f + t], c2))
        f += t
    return np.concatenate(out)


def _check(L, dev, orc, y1, c2, lens):
    want = _want(orc, y1, c2, lens)
    for engine in (True, False):
        got = _run(L, dev, y1, c2, lens, engine)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32),
                                      err_msg=f"{'position-pair' if engine else 'lane-pair'} kernel")


@pytest.mark.parametrize("t", [5, 6, 9, 10, 11, 57, 400])
def test_conv2_one_window(gpu_lib, dev, orc, t):
    rng = np.random.default_rng(t)
    _check(gpu_lib, dev, orc, _y1(rng, t), _c2(rng), [t])


def test_conv2_stacked_windows(gpu_lib, dev, orc):
    rng = np.random.default_rng(21)
    lens = [5, 12, 33, 7, 100, 9, 10]
    _check(gpu_lib, dev, orc, _y1(rng, sum(lens)), _c2(rng), lens)


def test_conv2_special_inputs(gpu_lib, dev, orc):
    """Negative inputs and signed zeros (the kernels take any fp32 input, not only ReLU output),
    a window of zeros, one non-zero input, subnormal products (|x w| near 1e-40) and products
    that overflow to infinity (ReLU of a NaN sum is 0 on both sides)."""
    rng = np.random.default_rng(22)
    c2 = _c2(rng)
    signed = rng.standard_normal((23, 32, 40)).astype(np.float32)
    signed[rng.random(signed.shape) < 0.2] = -0.0
    zeros = np.zeros((10, 32, 40), np.float32)
    one = np.zeros((15, 32, 40), np.float32)
    one[7, 3, 20] = 2.5
    _check(gpu_lib, dev, orc, signed, c2, [23])
    _check(gpu_lib, dev, orc, np.concatenate([zeros, one]), c2, [10, 15])
    tiny = _y1(rng, 17, 1e-20)
    _check(gpu_lib, dev, orc, tiny, _c2(rng, 1e-20), [17])
    huge = _y1(rng, 12, 1e30)
    _check(gpu_lib, dev, orc, huge, _c2(rng, 1e10), [12])


def _run_conv1(L, dev, x, c1, lens, by_value):
    frames = x.shape[0]
    py1 = dev.put(np.full((frames, 32, 40), np.nan, np.float32))
    if len(lens) == 1:
        rc = L.wasr_conv1(dev.put(x), dev.put(c1), None, 0, frames, by_value, py1, None)
    else:
        foff = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        rc = L.wasr_conv1(dev.put(x), dev.put(c1), dev.put(foff), len(lens), frames, by_value, py1, None)
    assert rc == 0
    return dev.get(py1, (frames, 32, 40), np.float32)


@pytest.mark.parametrize("lens", [[1], [2], [5], [57], [400], [5, 1, 13, 2, 7, 64, 3]])
def test_conv1(gpu_lib, dev, orc, lens):
    rng = np.random.default_rng(sum(lens) + len(lens))
    x = rng.standard_normal((sum(lens), 40)).astype(np.float32)
    x[rng.random(x.shape) < 0.05] = -0.0
    c1 = (rng.standard_normal((32, 1, 5, 5)) * 0.2).astype(np.float32)
    want, f = [], 0
    for t in lens:
        want.append(orc.conv1(x[f:f + t], c1))
        f += t
    want = np.concatenate(want)
    for by_value in (1, 0):
        got = _run_conv1(gpu_lib, dev, x, c1, lens, by_value)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32),
                                      err_msg="weights by value" if by_value else "weights from memory")
