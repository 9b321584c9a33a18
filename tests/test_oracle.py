"""CPU tests of the oracle (the C restatement of the reference CPU path) against the
reference's own known-answer test and against independent numpy / torch restatements.

Pins: src/kernels.rs:185-208 (qgemm_matches_scalar, reproduced bit for bit including its
LCG), exact int32 accumulators against an int64 numpy matmul, and each float op against a
straightforward float32/float64 numpy evaluation in the documented order.
"""
import numpy as np
import pytest


def lcg_stream(seed=7):
    """The LCG of src/kernels.rs:192-196: seed = seed*1103515245 + 12345 (wrapping u32);
    value = (seed >> 16) as i32 % 255 - 127."""
    s = seed
    while True:
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        yield (s >> 16) % 255 - 127


def kat0_inputs():
    t, k, n = 5, 64, 11
    r = lcg_stream(7)
    x = np.array([next(r) for _ in range(t * k)], np.float32) * np.float32(0.01)
    w = np.array([next(r) for _ in range(n * k)], np.int64).astype(np.int8)
    b = np.arange(n, dtype=np.float32)
    return t, k, n, x.reshape(t, k), w.reshape(n, k), b


def np_quant(x):
    """src/kernels.rs:11-25 in numpy float32 (half-away rounding done exactly in float64)."""
    x = np.asarray(x, np.float32)
    m = np.max(np.abs(x), axis=1)
    sc = np.where(m > 0, (m / np.float32(127.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / sc).astype(np.float32)
    v = (x * inv[:, None]).astype(np.float32).astype(np.float64)
    q = np.sign(v) * np.floor(np.abs(v) + 0.5)
    return np.clip(q, -127, 127).astype(np.int8), sc


def test_kat0_qgemm_matches_scalar(orc):
    """src/kernels.rs:185-208, reproduced: qgemm vs scalar dot1 within 1e-3 relative."""
    t, k, n, x, w, b = kat0_inputs()
    q, s = orc.quant(x)
    out = orc.qgemm(q, s, w, 0.5, bias=b)
    for i in range(t):
        for j in range(n):
            e = np.float32(orc.dot1(q[i], w[j])) * s[i] * np.float32(0.5) + b[j]
            assert abs(out[i, j] - e) <= 1e-3 * max(abs(e), 1.0), (i, j)
    # the golden fixture committed from this KAT (tests/golden/make_golden.py) still matches
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat0.npz"))
    np.testing.assert_array_equal(g["x"], x)
    np.testing.assert_array_equal(g["w"], w)
    np.testing.assert_array_equal(g["q"], q)
    np.testing.assert_array_equal(g["s"], s)
    np.testing.assert_array_equal(g["out"], out)


def test_quant_matches_numpy(orc):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((257, 512)).astype(np.float32)
    x[3] = 0.0                    # all-zero row -> scale 1
    x[4, :] = 0.5                 # exact .5 ties after scaling
    x[5, 7] = 1e-30               # tiny
    q, s = orc.quant(x)
    q2, s2 = np_quant(x)
    np.testing.assert_array_equal(s, s2)
    np.testing.assert_array_equal(q, q2)
    assert s[3] == 1.0 and not q[3].any()
    assert q.max() <= 127 and q.min() >= -127


def test_quant_ties_round_half_away(orc):
    # values whose scaled result is exactly k + 0.5 must round away from zero (Rust f32::round)
    x = np.array([[127.0, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 0.0]], np.float32)
    q, s = orc.quant(x)
    assert s[0] == 1.0
    assert list(q[0]) == [127, 1, -1, 2, -2, 3, -3, 0]


def test_quant_nan_and_inf_like_rust(orc):
    """Rust's `(v * inv).round().clamp(-127.0, 127.0) as i8` (src/kernels.rs:20): NaN stays NaN
    through clamp and `as i8` makes it 0; +-inf clamps to +-127.  The row max ignores NaN
    (f32::max), and an infinite max makes inv = 0, so every value of that row becomes
    NaN or 0 -> 0."""
    x = np.array([[np.nan, 1.0, -2.0, 0.5], [np.inf, 3.0, -np.inf, np.nan], [np.nan, np.nan, 0.0, 0.0]],
                 np.float32)
    q, s = orc.quant(x)
    assert q[0].tolist() == [0, 64, -127, 32] and s[0] == np.float32(2.0) / np.float32(127.0)
    assert q[1].tolist() == [0, 0, 0, 0] and np.isinf(s[1])
    assert q[2].tolist() == [0, 0, 0, 0] and s[2] == 1.0


@pytest.mark.parametrize("shape", [(400, 512, 2048), (37, 2048, 512), (64, 3840, 512), (3, 512, 10502)])
def test_qgemm_int32_exact_and_epilogue(orc, shape):
    """Config-0 style GEMM: AVX2 dot2x4 path == scalar dot1 == int64 numpy; epilogue equals
    ((acc*xs)*ws[j] + b[j]) evaluated in float32, bit for bit."""
    t, k, n = shape
    rng = np.random.default_rng(t + k + n)
    a = rng.standard_normal((t, k)).astype(np.float32)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    b = (0.02 * rng.standard_normal(n)).astype(np.float32)
    q, s = orc.quant(a)
    acc_np = (q.astype(np.int64) @ w.astype(np.int64).T)
    assert np.abs(acc_np).max() < 2 ** 31
    acc = orc.qgemm_acc(q, w)
    np.testing.assert_array_equal(acc, acc_np.astype(np.int32))
    out = orc.qgemm(q, s, w, 0.0, ws_vec=ws, bias=b)
    ref = ((acc_np.astype(np.float32) * s[:, None]).astype(np.float32) * ws[None, :]).astype(np.float32) + b[None, :]
    np.testing.assert_array_equal(out, ref.astype(np.float32))
    out2 = orc.qgemm(q, s, w, 0.0123)
    ref2 = ((acc_np.astype(np.float32) * s[:, None]).astype(np.float32) * np.float32(0.0123)).astype(np.float32)
    np.testing.assert_array_equal(out2, ref2 + np.float32(0.0))


def seq_sum_rows(x):
    s = np.zeros(x.shape[0], np.float32)
    for j in range(x.shape[1]):
        s = (s + x[:, j]).astype(np.float32)
    return s


def test_norm_matches_sequential_numpy(orc):
    rng = np.random.default_rng(3)
    x = (3.0 * rng.standard_normal((64, 512)) + 1.0).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    b = (0.05 * rng.standard_normal(512)).astype(np.float32)
    y = orc.norm(x, g, b)
    m = (seq_sum_rows(x) / np.float32(512.0)).astype(np.float32)
    d = (x - m[:, None]).astype(np.float32)
    v = (seq_sum_rows((d * d).astype(np.float32)) / np.float32(512.0)).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt((v + np.float32(1e-6)).astype(np.float32))).astype(np.float32)
    ref = ((d * inv[:, None]).astype(np.float32) * g).astype(np.float32) + b
    np.testing.assert_array_equal(y, ref.astype(np.float32))


def test_gelu_close_to_float64(orc):
    x = np.linspace(-8, 8, 2001).astype(np.float32)
    y = orc.gelu(x)
    xd = x.astype(np.float64)
    ref = 0.5 * xd * (1 + np.tanh(0.7978846 * (xd + 0.044715 * xd ** 3)))
    # float32 cancellation for x << 0 gives -0.0 where float64 has ~1e-7: absolute floor
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)


def test_attention_close_to_float64(orc):
    rng = np.random.default_rng(5)
    t = 77
    q, k, v = [rng.standard_normal((t, 512)).astype(np.float32) for _ in range(3)]
    out = orc.attention(q, k, v)
    ref = np.zeros((t, 512))
    for h in range(8):
        sl = slice(h * 64, (h + 1) * 64)
        s = q[:, sl].astype(np.float64) @ k[:, sl].astype(np.float64).T * 0.125
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        ref[:, sl] = p @ v[:, sl].astype(np.float64)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-5)


def test_frontend_matches_torch_conv(orc):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    t = 63
    x = rng.standard_normal((t, 40)).astype(np.float32)
    c1 = rng.standard_normal((32, 1, 5, 5)).astype(np.float32) * 0.3
    c2 = rng.standard_normal((64, 32, 7, 7)).astype(np.float32) * 0.03
    c3 = rng.standard_normal((192, 64, 3, 3)).astype(np.float32) * 0.05
    y3 = orc.frontend(x, c1, c2, c3)
    t1 = (t - 5) // 5 + 1
    X = torch.from_numpy(x).double()[None, None]
    y1 = torch.relu(torch.nn.functional.conv2d(X, torch.from_numpy(c1).double(), padding=2))
    y2 = torch.relu(torch.nn.functional.conv2d(y1, torch.from_numpy(c2).double(), stride=(5, 1), padding=(1, 3)))
    y2 = torch.nn.functional.pad(y2, (0, 1))          # column 40 = 0
    y3r = torch.relu(torch.nn.functional.conv2d(y2, torch.from_numpy(c3).double(), stride=(1, 2), padding=(1, 0)))
    # [1][192][t1][20] -> [t1][192*20]
    y3r = y3r[0].permute(1, 0, 2).reshape(y3r.shape[2], -1).numpy()
    assert y3.shape == (t1, 3840) and y3r.shape[0] == t1
    np.testing.assert_allclose(y3, y3r, rtol=1e-4, atol=1e-4)


def test_conv1_stage_matches_torch_conv(orc):
    """The conv1 stage alone (the checker of the GPU conv1 kernels), on windows of 1, 2 and 57
    frames (padding 2 in time and frequency)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(11)
    c1 = rng.standard_normal((32, 1, 5, 5)).astype(np.float32) * 0.3
    for t in (1, 2, 57):
        x = rng.standard_normal((t, 40)).astype(np.float32)
        y1 = orc.conv1(x, c1)
        ref = torch.relu(torch.nn.functional.conv2d(torch.from_numpy(x).double()[None, None],
                                                    torch.from_numpy(c1).double(), padding=2))
        ref = ref[0].permute(1, 0, 2).numpy()                           # [t][32][40]
        assert y1.shape == (t, 32, 40)
        np.testing.assert_allclose(y1, ref, rtol=1e-5, atol=1e-5)


def test_conv2_stage_matches_torch_conv(orc):
    """The conv2 stage alone (the checker of the GPU conv2 kernels), incl. a window of fewer
    than 5 frames (no output rows) and the zero column 40."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(10)
    c2 = rng.standard_normal((64, 32, 7, 7)).astype(np.float32) * 0.03
    assert orc.conv2(np.ones((4, 32, 40), np.float32), c2).shape == (0, 64, 41)
    for t in (5, 9, 10, 37):
        y1 = np.maximum(rng.standard_normal((t, 32, 40)), 0.0).astype(np.float32)
        y2 = orc.conv2(y1, c2)
        Y1 = torch.from_numpy(y1).double().permute(1, 0, 2)[None]      # [1][32][t][40]
        y2r = torch.relu(torch.nn.functional.conv2d(Y1, torch.from_numpy(c2).double(), stride=(5, 1),
                                                    padding=(1, 3)))
        y2r = y2r[0].permute(1, 0, 2).numpy()                           # [t1][64][40]
        assert y2.shape == ((t - 5) // 5 + 1, 64, 41)
        assert not y2[:, :, 40].any()
        np.testing.assert_allclose(y2[:, :, :40], y2r, rtol=1e-4, atol=1e-4)


def test_fbank_frame_matches_numpy_fft(orc):
    rng = np.random.default_rng(11)
    x = rng.integers(-20000, 20000, size=400).astype(np.int16)
    out = orc.fbank_frame(x)
    xd = x.astype(np.float64)
    pe = np.concatenate([[xd[0] * (1 - 0.97)], xd[1:] - 0.97 * xd[:-1]])
    ham = 0.54 - 0.46 * np.cos(2 * np.pi * np.arange(400) / 399)
    spec = np.fft.fft(np.concatenate([pe * ham, np.zeros(112)]))
    p = np.abs(spec[1:257]) ** 2
    mel = lambda f: 1127.0 * np.log(1 + f / 700.0)  # noqa: E731
    cf = mel(8000.0) * np.arange(1, 41) / 40
    ref = np.zeros(40)
    for kk in range(1, 257):
        m = mel(kk * 16000.0 / 512)
        c = int(np.sum(cf < m))
        if c == 0:
            ref[0] += p[kk - 1] * m / cf[0]
        elif c < 39:
            w = (cf[c] - m) / (cf[c] - cf[c - 1])
            ref[c - 1] += p[kk - 1] * w
            ref[c] += p[kk - 1] * (1 - w)
        elif c == 39:
            ref[38] += p[kk - 1] * (cf[39] - m) / (cf[39] - cf[38])
    ref[:39] = np.log(np.maximum(ref[:39], 1.0))
    ref[39] = np.log(max(np.sum(xd * xd), 1e-10))
    np.testing.assert_allclose(out, ref, rtol=1e-9, atol=1e-9)


def test_fbank_cms_and_silence(orc):
    rng = np.random.default_rng(12)
    pcm = rng.integers(-3000, 3000, size=16000).astype(np.int16)
    feats, sil = orc.fbank(pcm)
    n = (16000 - 400) // 160 + 1
    assert feats.shape == (n, 40)
    raw = np.stack([orc.fbank_frame(pcm[k * 160:k * 160 + 400]) for k in range(n)])
    for k in (0, 1, 49, 50, 51, n - 1):
        lo = max(0, k - 49)
        ref = (raw[k] - raw[lo:k + 1].sum(0) / (k + 1 - lo)).astype(np.float32)
        np.testing.assert_allclose(feats[k], ref, rtol=1e-6, atol=1e-5)
    s = np.zeros(40)
    s[39] = np.log(1e-10)
    np.testing.assert_allclose(sil, (s - raw[n - 50:].sum(0) / 50).astype(np.float32), rtol=1e-6, atol=1e-4)
    # short input: fewer than 400 samples gives no frame
    f2, _ = orc.fbank(pcm[:399])
    assert f2.shape[0] == 0


def test_ctc(orc):
    ids = np.array([0, 3, 3, 0, 3, 5, 5, 5, 0, 0, 7], np.uint32)
    assert list(orc.ctc(ids)) == [3, 3, 5, 7]
    assert list(orc.ctc(np.zeros(4, np.uint32))) == []
