"""The oracle pinned against the reference itself: the reference's own CUDA library
(csrc/wtlgpu.cu, csrc/wtl_kern.cu, csrc/wk_attention_*.cu), compiled unmodified from its sources
by oracle/Makefile into oracle/_ref/libwasr_ref.so, runs beside the oracle on the same inputs.

The reference's GPU path is not bit-identical to its own CPU path (its header says so:
csrc/wtl_kern.cu:9-10): nvcc contracts its sums into FMAs, its attention runs on cuBLAS SGEMM
with __expf, its GELU calls CUDA's tanhf.  So the pins come in two strengths:

* exact, where the reference's GPU arithmetic is exact or in the CPU's order: the int32
  accumulators of the cuBLASLt int8 GEMM (read through wp_gemm with unit scales), the per-row
  quantisation (csrc/wtl_kern.cu:218-242), the argmax with its first-max-wins ties
  (csrc/wtl_kern.cu:282-306), the residual add;
* within a stated tolerance elsewhere -- tight enough that a wrong tap, stride, pad, scale,
  operand or reduction order in the oracle shows up, loose enough for FMA contraction and
  library exp / tanh: the dequantising GEMM epilogue, LayerNorm+quant, GELU+quant, the conv
  frontend, attention, and the fused GEMM+quant entry points.

Every comparison is oracle vs reference; the B200 library equals the oracle bit for bit in the
other test files, so these pins carry over to it (and the exact ones are checked directly too).
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libwasr_ref.so")
P, I, Z, F = C.c_void_p, C.c_int, C.c_size_t, C.c_float
NONE = C.c_size_t(-1).value


@pytest.fixture(scope="module")
def ref(gpu_lib, tmp_path_factory):
    assert os.path.exists(REF_SO), "oracle/_ref/libwasr_ref.so is missing: `make -C oracle ref` builds it"
    # the reference keeps a cuBLASLt algorithm cache on disk: keep it inside the test's tmp dir
    os.environ["WTL_ALGO_CACHE"] = str(tmp_path_factory.mktemp("ref_cache") / "lt_algo.bin")
    os.environ.pop("WTL_ATTN_MATH", None)   # full fp32 SGEMM, the reference's default
    os.environ.pop("WTL_ATTN_IMPL", None)   # cuBLAS attention, the reference's default
    L = C.CDLL(REF_SO, mode=os.RTLD_LOCAL)
    sig = {
        "wp_create": (P, [P, Z]), "wp_destroy": (None, [P]), "wp_sync": (I, [P]),
        "wp_gemm": (I, [P, P, P, I, I, Z, I, F, Z, P]),
        "wp_gemm_q": (I, [P, P, P, I, I, Z, I, F, P, P, P, P]),
        "wp_gemm_qg": (I, [P, P, P, I, I, Z, I, F, P, P, P, P]),
        "wk_front": (None, [P, P, P, P, P, I, I, P, P, P]),
        "wk_norm_quant": (None, [P, P, P, P, I, I, P, P]),
        "wk_add_norm_quant": (None, [P, P, P, P, P, I, I, P, P]),
        "wk_quant": (None, [P, P, I, I, P, P]),
        "wk_gelu_quant": (None, [P, P, I, I, P, P]),
        "wk_argmax": (None, [P, P, I, I, P]),
        "wk_attention_fast": (I, [P, P, P, P, I, I, I, P, P]),
        "wk_last_error": (I, []),
    }
    for k, (r, a) in sig.items():
        f = getattr(L, k)
        f.restype, f.argtypes = r, a
    return L


def _ref_ctx(R, mats):
    """A context of library R (the reference's or the B200 one: both export wp_create) over
    matrices packed 256-byte aligned (build_plan's rule)."""
    parts, offs, size = [], [], 0
    for a in mats:
        pad = (-size) % 256
        parts.append(b"\0" * pad)
        size += pad
        offs.append(size)
        b = np.ascontiguousarray(a).tobytes()
        parts.append(b)
        size += len(b)
    blob = np.frombuffer(b"".join(parts), np.uint8).copy()
    ctx = R.wp_create(blob.ctypes.data, blob.size)
    assert ctx, "wp_create failed"
    return ctx, offs


@pytest.fixture()
def rctx(ref):
    """A small reference context whose legacy-stream wp_sync orders the wk_* calls."""
    ctx, _ = _ref_ctx(ref, [np.zeros((4, 64), np.int8)])
    yield ctx
    ref.wp_destroy(ctx)


def test_gemm_int32_accumulators_exact(ref, gpu_lib, dev, orc):
    """cuBLASLt int8 accumulators (csrc/wtlgpu.cu:574) = the oracle's qgemm accumulators
    (src/kernels.rs:33-85): read through wp_gemm with xs = 1, ws = 1, no bias, where the
    reference's epilogue reduces to (float)acc, the same conversion the CPU makes."""
    rng = np.random.default_rng(21)
    for t, k, n in [(300, 512, 2048), (133, 3840, 512), (257, 2048, 512), (64, 512, 1536)]:
        xq = rng.integers(-127, 128, size=(t, k), dtype=np.int8)
        w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        ctx, offs = _ref_ctx(ref, [w])
        try:
            pq, ps, po = dev.put(xq), dev.put(np.ones(t, np.float32)), dev.empty(t * n * 4)
            assert ref.wp_gemm(ctx, pq, ps, t, k, offs[0], n, 1.0, NONE, po) == 0
            assert ref.wp_sync(ctx) == 0
            got = dev.get(po, (t, n), np.float32)
        finally:
            ref.wp_destroy(ctx)
        acc = orc.qgemm_acc(xq, w)
        np.testing.assert_array_equal(got, acc.astype(np.float32), err_msg=f"{t}x{k}x{n}")
        # and the B200 library's raw accumulators
        ours, offs2 = _ref_ctx(gpu_lib, [w])
        try:
            pi = dev.empty(t * n * 4)
            assert gpu_lib.wp_gemm_i32(ours, pq, t, k, offs2[0], n, None, pi) == 0
            assert gpu_lib.wp_sync(ours) == 0
            np.testing.assert_array_equal(dev.get(pi, (t, n), np.int32), acc)
        finally:
            gpu_lib.wp_destroy(ours)


def test_gemm_epilogue_within_fma_rounding(ref, dev, orc):
    """wp_gemm's dequantising epilogue (csrc/wtlgpu.cu:249-257) computes acc * (xs * ws) + bias,
    which nvcc contracts into one FMA; the CPU computes (acc * xs) * ws + bias (src/kernels.rs:53).
    They agree to a few units in the last place of acc * xs * ws."""
    rng = np.random.default_rng(22)
    t, k, n = 200, 512, 2048
    x = rng.standard_normal((t, k)).astype(np.float32)
    xq, xs = orc.quant(x)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    b = (0.3 * rng.standard_normal(n)).astype(np.float32)
    ws = np.float32(1.0 / (73.6 * np.sqrt(k)))
    ctx, offs = _ref_ctx(ref, [w, b])
    try:
        pq, ps, po = dev.put(xq), dev.put(xs), dev.empty(t * n * 4)
        assert ref.wp_gemm(ctx, pq, ps, t, k, offs[0], n, float(ws), offs[1], po) == 0
        assert ref.wp_sync(ctx) == 0
        got = dev.get(po, (t, n), np.float32)
    finally:
        ref.wp_destroy(ctx)
    want = orc.qgemm(xq, xs, w, ws, bias=b)
    prod = np.abs(orc.qgemm_acc(xq, w).astype(np.float64) * xs[:, None] * float(ws))
    assert np.all(np.abs(got.astype(np.float64) - want) <= 4 * np.spacing(np.float32(prod + np.abs(b)))), \
        "epilogue differs by more than FMA rounding"


@pytest.mark.parametrize("k", [512, 2048, 3840])
def test_quant_exact(ref, rctx, gpu_lib, dev, orc, k):
    """Per-row dynamic quantisation (csrc/wtl_kern.cu:218-242 = src/kernels.rs:11-25): scale
    max|x| / 127 (1 for an all-zero row), q = roundf(x * (1 / s)) clamped to +-127, half away
    from zero -- identical on every value, exact .5 ties and zero rows included."""
    rng = np.random.default_rng(k)
    t = 97
    x = (rng.standard_normal((t, k)) * rng.uniform(0.01, 50, size=(t, 1))).astype(np.float32)
    x[0, :8] = [0.5, -0.5, 1.5, 127, -127, 0.25, 2.5, -2.5]   # s = 1: exact ties
    x[3] = 0.0
    px, pq, ps = dev.put(x), dev.empty(t * k), dev.empty(t * 4)
    ref.wk_quant(None, px, t, k, pq, ps)
    assert ref.wp_sync(rctx) == 0 and ref.wk_last_error() == 0
    q, s = orc.quant(x)
    np.testing.assert_array_equal(dev.get(ps, (t,), np.float32), s)
    np.testing.assert_array_equal(dev.get(pq, (t, k), np.int8), q)
    gpu_lib.wk_quant(None, px, t, k, pq, ps)                 # the B200 library, same bits
    np.testing.assert_array_equal(dev.get(pq, (t, k), np.int8), q)


def test_argmax_exact(ref, rctx, dev, orc):
    """argmax with first-max-wins ties (csrc/wtl_kern.cu:282-306 = src/model.rs:499-500)."""
    rng = np.random.default_rng(23)
    t, n = 64, 10504
    x = rng.standard_normal((t, n)).astype(np.float32)
    x[0, :] = 1.0
    x[1, 17], x[1, 9000] = 9.0, 9.0
    x[2, 10502:] = -1e30
    px, po = dev.put(x), dev.empty(t * 4)
    ref.wk_argmax(None, px, t, n, po)
    assert ref.wp_sync(rctx) == 0 and ref.wk_last_error() == 0
    want = np.array([orc.lib().wo_argmax(x[i].ctypes.data, n) for i in range(t)], np.uint32)
    np.testing.assert_array_equal(dev.get(po, (t,), np.uint32), want)


def _ln_inputs(t, seed):
    rng = np.random.default_rng(seed)
    h = (4 * rng.standard_normal((t, 512)) + 0.3).astype(np.float32)
    o = rng.standard_normal((t, 512)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    b = (0.05 * rng.standard_normal(512)).astype(np.float32)
    return h, o, g, b


def _close_quant(got_q, got_s, want_q, want_s):
    # a scale one ulp off moves a value across a rounding boundary only rarely
    np.testing.assert_allclose(got_s, want_s, rtol=1e-6)
    d = np.abs(got_q.astype(np.int32) - want_q.astype(np.int32))
    assert d.max() <= 1 and np.mean(d == 0) >= 0.999, (d.max(), np.mean(d == 0))


def test_layernorm_quant_within_fma_rounding(ref, rctx, dev, orc):
    """norm_quant / add_norm_quant (csrc/wtl_kern.cu:124-216): mean by a sequential sum, biased
    variance, (x - m) * inv * g + b, then the row quant -- the CPU's order (src/model.rs:693-704)
    except that nvcc contracts the variance sum into FMAs.  The residual add is exact."""
    t = 300
    h, o, g, b = _ln_inputs(t, 24)
    ph, po, pg, pb = dev.put(h), dev.put(o), dev.put(g), dev.put(b)
    pq, ps = dev.empty(t * 512), dev.empty(t * 4)
    ref.wk_norm_quant(None, ph, pg, pb, t, 512, pq, ps)
    assert ref.wp_sync(rctx) == 0
    q, s = orc.quant(orc.norm(h, g, b))
    _close_quant(dev.get(pq, (t, 512), np.int8), dev.get(ps, (t,), np.float32), q, s)
    ref.wk_add_norm_quant(None, ph, po, pg, pb, t, 512, pq, ps)
    assert ref.wp_sync(rctx) == 0 and ref.wk_last_error() == 0
    h2 = (h + o).astype(np.float32)
    np.testing.assert_array_equal(dev.get(ph, (t, 512), np.float32), h2)
    q, s = orc.quant(orc.norm(h2, g, b))
    _close_quant(dev.get(pq, (t, 512), np.int8), dev.get(ps, (t,), np.float32), q, s)


def test_gelu_quant_within_tanhf_error(ref, rctx, dev, orc):
    """gelu_quant (csrc/wtl_kern.cu:245-275): the GELU formula of src/model.rs:710-712 with
    explicitly rounded products, on CUDA's tanhf (a couple of ulps from glibc's): the GELU values
    agree to that error, the quantised rows to one step."""
    rng = np.random.default_rng(25)
    t, k = 256, 2048
    x = (2 * rng.standard_normal((t, k))).astype(np.float32)
    px, pq, ps = dev.put(x), dev.empty(t * k), dev.empty(t * 4)
    ref.wk_gelu_quant(None, px, t, k, pq, ps)
    assert ref.wp_sync(rctx) == 0 and ref.wk_last_error() == 0
    got = dev.get(px, (t, k), np.float32)
    want = orc.gelu(x)
    # 1 + tanh(u) cancels for large negative x: bound the error by the input's magnitude
    assert np.all(np.abs(got - want) <= 4e-7 * np.maximum(np.abs(x), 1.0))
    q, s = orc.quant(want)
    _close_quant(dev.get(pq, (t, k), np.int8), dev.get(ps, (t,), np.float32), q, s)


@pytest.mark.parametrize("t", [9, 390, 1950])
def test_frontend_within_fma_rounding(ref, rctx, dev, orc, pkg, t):
    """The conv frontend (csrc/wtl_kern.cu:46-120 = src/model.rs:389-478): same taps, padding,
    strides, the 41st zero column and ReLUs; the reference sums each output with FMAs in two
    interleaved partial sums, the CPU in dotf's 8 lanes, so y3 agrees to float rounding."""
    blob, plan = pkg.synth.make_model(seed=3, n_layers=1)
    c1 = np.frombuffer(blob, np.float32, 32 * 25, plan.c1)
    c2 = np.frombuffer(blob, np.float32, 64 * 1568, plan.c2)
    c3 = np.frombuffer(blob, np.float32, 192 * 576, plan.c3)
    feats, _ = pkg.fbank(pkg.synth.make_audio(30 + t, (t + 2) * 0.01 + 0.015))
    x = np.ascontiguousarray(feats[:t])
    assert x.shape[0] == t
    t1 = (t - 5) // 5 + 1
    px, p1, p2, p3 = dev.put(x), dev.put(c1), dev.put(c2), dev.put(c3)
    y1, y2, y3 = dev.empty(t * 1280 * 4), dev.empty(t1 * 2624 * 4), dev.empty(t1 * 3840 * 4)
    ref.wk_front(None, px, p1, p2, p3, t, t1, y1, y2, y3)
    assert ref.wp_sync(rctx) == 0 and ref.wk_last_error() == 0
    got = dev.get(y3, (t1, 3840), np.float32)
    want = orc.frontend(x, c1, c2, c3)
    scale = float(np.max(np.abs(want)))
    assert scale > 0
    err = float(np.max(np.abs(got - want))) / scale
    assert err <= 1e-5, err
    # ReLU zeros and the flatten order agree exactly where the values are clear of zero
    clear = np.abs(want) > 1e-4 * scale
    np.testing.assert_array_equal(got[clear] > 0, want[clear] > 0)


@pytest.mark.parametrize("t", [13, 150, 390])
def test_attention_within_library_rounding(ref, rctx, dev, orc, t):
    """Attention (csrc/wk_attention_cublas.cu:78-117, the reference's default): scores
    0.125 * q.k per head of 64, softmax over the keys, probabilities times v -- the math of
    src/model.rs:714-739 on cuBLAS SGEMM and __expf, so within library rounding."""
    rng = np.random.default_rng(t + 7)
    q, k, v = [(rng.standard_normal((t, 512)) * 1.5).astype(np.float32) for _ in range(3)]
    pq, pk, pv, po = dev.put(q), dev.put(k), dev.put(v), dev.empty(t * 512 * 4)
    sc = dev.empty(8 * t * t * 4)
    assert ref.wk_attention_fast(None, pq, pk, pv, t, 512, 8, sc, po) == 0
    assert ref.wp_sync(rctx) == 0 and ref.wk_last_error() == 0
    got = dev.get(po, (t, 512), np.float32)
    want = orc.attention(q, k, v)
    err = float(np.max(np.abs(got - want))) / float(np.max(np.abs(want)))
    assert err <= 1e-4, err


def test_gemm_requant_entry_points(ref, dev, orc):
    """wp_gemm_q / wp_gemm_qg (csrc/wtlgpu.cu:264-341): epilogue, optional GELU and the row
    quant in one call -- within one int8 step of the oracle's quant(qgemm) / quant(gelu(qgemm))."""
    rng = np.random.default_rng(26)
    t, k, n = 300, 512, 2048
    x = rng.standard_normal((t, k)).astype(np.float32)
    xq, xs = orc.quant(x)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    b = (0.3 * rng.standard_normal(n)).astype(np.float32)
    ws = np.float32(1.0 / (73.6 * np.sqrt(k)))
    ctx, offs = _ref_ctx(ref, [w])
    try:
        pq, ps, pb = dev.put(xq), dev.put(xs), dev.put(b)
        oq, osc = dev.empty(t * n), dev.empty(t * 4)
        y = orc.qgemm(xq, xs, w, ws, bias=b)
        for fn, f in ((ref.wp_gemm_q, lambda a: a), (ref.wp_gemm_qg, orc.gelu)):
            assert fn(ctx, pq, ps, t, k, offs[0], n, float(ws), pb, None, oq, osc) == 0
            assert ref.wp_sync(ctx) == 0
            q, s = orc.quant(f(y))
            _close_quant(dev.get(oq, (t, n), np.int8), dev.get(osc, (t,), np.float32), q, s)
    finally:
        ref.wp_destroy(ctx)
