"""GPU parity of the wk_* kernels (reference ABI, csrc/wtl_kern.cu / csrc/wk_attention_*.cu)
against the oracle, bit for bit: quant, LayerNorm+quant, add+LayerNorm+quant, add, argmax, the
conv frontend, GELU+quant and attention all follow the operation order of src/model.rs /
src/kernels.rs, and GELU and attention evaluate restatements of glibc's tanhf / expf."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_wk_quant_nan_inf_like_rust(gpu_lib, dev, orc):
    """NaN -> 0 and +-inf -> +-127 as Rust's clamp + `as i8` give them (src/kernels.rs:20), on the
    vectorised 512-wide path and the general path."""
    L = gpu_lib
    for k in (512, 1000):
        x = np.random.default_rng(k).standard_normal((3, k)).astype(np.float32)
        x[0, 0], x[0, 7] = np.nan, np.nan                     # NaN in a finite row
        x[1, 3], x[1, 5], x[1, 9] = np.inf, -np.inf, np.nan   # an infinite row max: inv = 0
        x[2, 1] = np.nan
        px, pq, ps = dev.put(x), dev.empty(3 * k), dev.empty(12)
        L.wk_quant(None, px, 3, k, pq, ps)
        assert L.wk_last_error() == 0
        q, s = orc.quant(x)
        got = dev.get(pq, (3, k), np.int8)
        np.testing.assert_array_equal(got, q)
        assert got[0, 0] == 0 and got[0, 7] == 0 and not got[1].any()
        np.testing.assert_array_equal(dev.get(ps, (3,), np.float32), s)


@pytest.mark.parametrize("t,k", [(1, 512), (390, 512), (77, 2048), (129, 3840), (5, 10), (3, 1000)])
def test_wk_quant(gpu_lib, dev, orc, t, k):
    L = gpu_lib
    rng = np.random.default_rng(t * k)
    x = (rng.standard_normal((t, k)) * rng.uniform(0.01, 100)).astype(np.float32)
    x[0, : min(k, 8)] = [0.5, -0.5, 1.5, 127, -127, 0.25, 3.0, -2.5][: min(k, 8)]
    if t > 2:
        x[2] = 0.0
    px, pq, ps = dev.put(x), dev.empty(t * k), dev.empty(t * 4)
    L.wk_quant(None, px, t, k, pq, ps)
    assert L.wk_last_error() == 0
    q, s = orc.quant(x)
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32), s)
    np.testing.assert_array_equal(dev.get(pq, (t, k), np.int8), q)
    # wp_quant_rows: same rounding
    assert L.wp_quant_rows(px, t, k, None, pq, ps) == 0
    np.testing.assert_array_equal(dev.get(pq, (t, k), np.int8), q)


@pytest.mark.parametrize("t", [1, 31, 33, 390, 777])
def test_wk_norm_quant_and_add(gpu_lib, dev, orc, t):
    L = gpu_lib
    rng = np.random.default_rng(t)
    h = (4 * rng.standard_normal((t, 512)) + 0.3).astype(np.float32)
    o = rng.standard_normal((t, 512)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    b = (0.05 * rng.standard_normal(512)).astype(np.float32)
    ph, po, pg, pb = dev.put(h), dev.put(o), dev.put(g), dev.put(b)
    pq, ps = dev.empty(t * 512), dev.empty(t * 4)
    L.wk_norm_quant(None, ph, pg, pb, t, 512, pq, ps)
    q, s = orc.quant(orc.norm(h, g, b))
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32), s)
    np.testing.assert_array_equal(dev.get(pq, (t, 512), np.int8), q)
    L.wk_add_norm_quant(None, ph, po, pg, pb, t, 512, pq, ps)
    h2 = (h + o).astype(np.float32)
    np.testing.assert_array_equal(dev.get(ph, (t, 512), np.float32), h2)
    q, s = orc.quant(orc.norm(h2, g, b))
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32), s)
    np.testing.assert_array_equal(dev.get(pq, (t, 512), np.int8), q)
    L.wk_add(None, ph, po, t, 512)
    np.testing.assert_array_equal(dev.get(ph, (t, 512), np.float32), (h2 + o).astype(np.float32))
    assert L.wk_last_error() == 0


def test_wk_norm_quant_ties_and_non_finite(gpu_lib, dev, orc):
    """With g = 0 every normalised value is its bias, so biases of 127 and +-(k + 0.5) put exact
    .5 ties in every row (scale 1, round half away from zero); one row holds a NaN and one an
    infinity (the rows the kernel quantises element by element)."""
    L = gpu_lib
    t = 40
    rng = np.random.default_rng(3)
    h = rng.standard_normal((t, 512)).astype(np.float32)
    h[5, 17] = np.nan
    h[9, 100] = np.inf
    g = np.zeros(512, np.float32)
    b = np.round(rng.uniform(-126, 126, 512)).astype(np.float32) + np.float32(0.5)
    b[0] = 127.0
    b[1:9] = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5]
    ph, pg, pb = dev.put(h), dev.put(g), dev.put(b)
    pq, ps = dev.empty(t * 512), dev.empty(t * 4)
    L.wk_norm_quant(None, ph, pg, pb, t, 512, pq, ps)
    assert L.wk_last_error() == 0
    q, s = orc.quant(orc.norm(h, g, b))
    got = dev.get(pq, (t, 512), np.int8)
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32).view(np.uint32), s.view(np.uint32))
    np.testing.assert_array_equal(got, q)
    assert list(got[0, 1:9]) == [1, -1, 2, -2, 3, -3, 127, -127]


def test_wk_norm_quant_other_width(gpu_lib, dev, orc):
    L = gpu_lib
    t, d = 9, 200
    rng = np.random.default_rng(2)
    h = rng.standard_normal((t, d)).astype(np.float32)
    g, b = np.ones(d, np.float32), np.zeros(d, np.float32)
    ph, pg, pb, pq, ps = dev.put(h), dev.put(g), dev.put(b), dev.empty(t * d), dev.empty(t * 4)
    L.wk_norm_quant(None, ph, pg, pb, t, d, pq, ps)
    q, s = orc.quant(orc.norm(h, g, b))
    np.testing.assert_array_equal(dev.get(pq, (t, d), np.int8), q)
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32), s)


def test_wk_gelu_quant(gpu_lib, dev, orc):
    """In-place GELU + per-row quant: bit-exact (the kernel evaluates glibc's tanhf algorithm)."""
    L = gpu_lib
    t, k = 300, 2048
    rng = np.random.default_rng(4)
    x = (2 * rng.standard_normal((t, k))).astype(np.float32)
    px, pq, ps = dev.put(x), dev.empty(t * k), dev.empty(t * 4)
    L.wk_gelu_quant(None, px, t, k, pq, ps)
    gx = orc.gelu(x)
    np.testing.assert_array_equal(dev.get(px, (t, k), np.float32), gx)
    q, s = orc.quant(gx)
    np.testing.assert_array_equal(dev.get(pq, (t, k), np.int8), q)
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32), s)


@pytest.mark.parametrize("t,n", [(390, 10504), (7, 10502), (1, 3), (64, 257)])
def test_wk_argmax_first_max_wins(gpu_lib, dev, orc, t, n):
    L = gpu_lib
    rng = np.random.default_rng(n)
    x = rng.standard_normal((t, n)).astype(np.float32)
    x[0, :] = 1.0                      # all equal -> index 0
    if t > 1:
        x[1, 5] = 9.0
        x[1, n - 1] = 9.0              # tie -> lower index
    if n > 10502:
        x[:, 10502:] = -1e30           # padded vocabulary columns never win
    px, po = dev.put(x), dev.empty(t * 4)
    L.wk_argmax(None, px, t, n, po)
    ref = np.array([orc.lib().wo_argmax(x[i].ctypes.data, n) for i in range(t)], np.uint32)
    np.testing.assert_array_equal(dev.get(po, (t,), np.uint32), ref)


@pytest.mark.parametrize("t", [5, 9, 64, 1950, 2003])
def test_wk_front_bit_exact(gpu_lib, dev, orc, pkg, t):
    L = gpu_lib
    rng = np.random.default_rng(t)
    x = (3 * rng.standard_normal((t, 40))).astype(np.float32)
    c1 = (rng.standard_normal((32, 1, 5, 5)) * np.sqrt(2 / 25)).astype(np.float32)
    c2 = (rng.standard_normal((64, 32, 7, 7)) * np.sqrt(2 / 1568)).astype(np.float32)
    c3 = (rng.standard_normal((192, 64, 3, 3)) * np.sqrt(2 / 576)).astype(np.float32)
    t1 = (t - 5) // 5 + 1
    px, p1, p2, p3 = dev.put(x), dev.put(c1), dev.put(c2), dev.put(c3)
    y1, y2, y3 = dev.empty(t * 1280 * 4), dev.empty(t1 * 2624 * 4), dev.empty(t1 * 3840 * 4)
    L.wk_front(None, px, p1, p2, p3, t, t1, y1, y2, y3)
    assert L.wk_last_error() == 0
    got = dev.get(y3, (t1, 3840), np.float32)
    np.testing.assert_array_equal(got, orc.frontend(x, c1, c2, c3))


# t covers every key-tail width of a key chunk (1 to 4 groups of 8 in a 32-key chunk and 1 to 8
# in a 64-key one: t mod 64 = 1, 13, 22, 31, 33, 45, 63, 0 and 8-key boundaries), 1- to 8-tile
# segments (65 and 100: tiles of 33 and 50 rows; tiles whose last warp holds 1 to 7 rows) and the
# largest shapes
@pytest.mark.parametrize("t", [1, 5, 8, 13, 31, 32, 33, 45, 63, 64, 65, 100, 127, 128, 129, 150, 200, 265,
                               390, 512])
def test_wk_attention(gpu_lib, dev, orc, t):
    L = gpu_lib
    rng = np.random.default_rng(t + 100)
    q, k, v = [(rng.standard_normal((t, 512)) * 1.5).astype(np.float32) for _ in range(3)]
    pq, pk, pv, po, sc = dev.put(q), dev.put(k), dev.put(v), dev.empty(t * 512 * 4), dev.empty(8 * t * t * 4)
    assert L.wk_attention_fast(None, pq, pk, pv, t, 512, 8, sc, po) == 0
    got = dev.get(po, (t, 512), np.float32)
    ref = orc.attention(q, k, v)
    np.testing.assert_array_equal(got, ref)   # same order, same glibc expf algorithm
    # the reference's other attention entry points run the same kernel here: same bits
    for name, scratch in (("wk_attention_tiled", None), ("wk_attention_cublas", sc)):
        zero = np.zeros((t, 512), np.float32)
        assert L.wp_h2d(po, zero.ctypes.data, zero.nbytes) == 0
        assert getattr(L, name)(None, pq, pk, pv, t, 512, 8, scratch, po) == 0
        np.testing.assert_array_equal(dev.get(po, (t, 512), np.float32), ref, err_msg=name)
    # return codes of csrc/wk_attention_*.cu
    assert L.wk_attention_fast(None, None, pk, pv, t, 512, 8, sc, po) == -1
    assert L.wk_attention_fast(None, pq, pk, pv, t, 512, 7, sc, po) == -2
    assert L.wk_attention_fast(None, pq, pk, pv, t, 256, 8, sc, po) == -3
    assert L.wk_attention_tiled_tuned(None, pq, pk, pv, t, 512, 8, po, 12, 64) == -4


def _math_inputs():
    # every 251st float bit pattern (all magnitudes) + a dense grid over the ranges the model uses
    u = np.arange(0, 2 ** 32, 251, dtype=np.uint64).astype(np.uint32)
    x = u.view(np.float32)
    x = x[np.isfinite(x)]
    dense = np.linspace(-40.0, 40.0, 4_000_001, dtype=np.float32)
    return np.concatenate([x, dense, np.array([0x4202422f, 0xc27c65d9], np.uint32).view(np.float32)])


@pytest.mark.parametrize("fn,name", [(0, "tanhf"), (1, "expf"), (2, "gelu"), (4, "tanhf"), (5, "gelu")])
def test_device_libm_restatements_bit_exact(gpu_lib, dev, orc, fn, name):
    """The GELU and softmax kernels evaluate glibc's tanhf / expf algorithms (the functions the
    reference's Rust f32::tanh / f32::exp call): bit-identical to this host's glibc."""
    L = gpu_lib
    x = _math_inputs()
    if name == "expf":
        x = x[(x > -110) & (x < 89)]
    px, py = dev.put(x), dev.empty(x.nbytes)
    assert L.wasr_eval_math(fn, px, py, x.size, None) == 0
    got = dev.get(py, x.shape, np.float32)
    ref = {"tanhf": orc.libm_tanhf, "expf": orc.libm_expf, "gelu": orc.gelu}[name](x)
    bad = np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, (bad.size, x[bad[:5]], got[bad[:5]], ref[bad[:5]])


def test_softmax_division_exact(gpu_lib, dev):
    """The attention softmax divides each exp by its row sum through a reciprocal and Markstein's
    correction (numerators in [0, 1], row sums in [1, 2^24)); the quotient must be the correctly
    rounded IEEE quotient, which is what the reference's f32 division gives."""
    L = gpu_lib
    rng = np.random.default_rng(11)
    a = np.arange(0, 0x3F800001, 97, dtype=np.uint32).view(np.float32)          # every 97th float in [0, 1]
    a = np.concatenate([a, np.float32([0.0, 1.0, 2.0 ** -80, 2.0 ** -81, 1e-30, 1e-45, 0.5])])
    specials = np.float32([1.0, np.nextafter(np.float32(1), np.float32(2)), np.nextafter(np.float32(2), np.float32(1)),
                           2.0, 3.0, 7.0, 255.0, 256.0, 8191.5, 3.0 * 2 ** 20, 16777215.0])
    b = np.where(rng.random(a.size) < 0.5, rng.uniform(1.0, 8192.0, a.size).astype(np.float32),
                 specials[rng.integers(0, specials.size, a.size)]).astype(np.float32)
    x = np.empty(2 * a.size, np.float32)
    x[0::2], x[1::2] = a, b
    px, py = dev.put(x), dev.empty(x.nbytes)
    assert L.wasr_eval_math(6, px, py, x.size, None) == 0
    got = dev.get(py, x.shape, np.float32)[0::2]
    ref = (a / b).astype(np.float32)
    bad = np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, (bad.size, a[bad[:5]], b[bad[:5]], got[bad[:5]], ref[bad[:5]])
