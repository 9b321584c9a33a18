"""The certified GELU + quant kernel (the engine's GELU for the model's FF width of 2048).

The GELU output feeds only its row's int8 quantisation (src/model.rs:495-496 with quant,
src/kernels.rs:11-25), so the kernel evaluates an approximate GELU, takes the row maximum from the
exact GELU of the candidate elements and re-quantises from the exact GELU every element whose
scaled value lies within the error bound of a rounding boundary.  These tests check the bound on
every float input, and that the int8 rows and scales equal the oracle's quant(gelu(x)) bit for
bit, including rows built so that many elements sit next to a rounding boundary, rows whose
largest values nearly tie, and rows with non-finite or vanishing values.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

K = 2048


def _run(L, dev, x, exact):
    m = x.shape[0]
    px, pq, ps = dev.put(x), dev.empty(m * K), dev.empty(m * 4)
    assert L.wasr_gelu_quant(px, m, K, pq, ps, exact, None) == 0
    return dev.get(pq, (m, K), np.int8), dev.get(ps, (m,), np.float32)


def _check(L, dev, orc, x):
    q, s = _run(L, dev, x, 0)
    qe, se = _run(L, dev, x, 1)
    rq, rs = orc.quant(orc.gelu(x))
    np.testing.assert_array_equal(s.view(np.uint32), rs.view(np.uint32))
    np.testing.assert_array_equal(q, rq)
    np.testing.assert_array_equal(qe, rq)
    np.testing.assert_array_equal(se.view(np.uint32), rs.view(np.uint32))


def test_gelu_cert_bound_on_every_float(gpu_lib, dev):
    """On all 2^32 inputs: |gelu_fast(x) - gelu(x)| <= A + B |gelu_fast(x)| where both are finite;
    the approximation is non-finite wherever the exact GELU is; the exact GELU is non-decreasing
    on [0, inf] and at most 0.171 in magnitude below 0 (the kernel's exact row maximum)."""
    L = gpu_lib
    stats = dev.put(np.zeros(8, np.uint64))
    assert L.wasr_gelu_cert_scan(0, 1 << 32, stats, None) == 0
    st = dev.get(stats, (8,), np.uint64)
    f = st.view(np.float64)
    print(f"gelu cert scan: max |g~ - g| - B|g~| = {f[0]:.3e}; max rel err (|g~| >= 1/16) {f[4]:.3e}; "
          f"max abs err (|g~| < 1/16) {f[5]:.3e}; max |g| below 0 {f[7]:.6f}; "
          f"only-approx-non-finite inputs {int(st[3])}")
    assert int(st[1]) == 0, "exact GELU non-finite where the approximation is finite"
    assert int(st[2]) == 0, f"bound exceeded on {int(st[2])} inputs (worst excess {f[0]:.3e})"
    assert int(st[6]) == 0, f"exact GELU decreases between {int(st[6])} adjacent non-negative floats"
    assert f[7] <= 0.171, f"|gelu| below 0 reaches {f[7]}"


@pytest.mark.parametrize("sigma", [0.5, 1.0, 2.0, 4.0])
def test_gelu_cert_random_rows(gpu_lib, dev, orc, sigma):
    rng = np.random.default_rng(int(sigma * 10))
    x = (sigma * rng.standard_normal((1029, K))).astype(np.float32)
    _check(gpu_lib, dev, orc, x)


def _near_ties(orc, rng, inv, lo, hi, n_want, band=2e-5):
    """x in [lo, hi) whose exact GELU, scaled by inv, lies within `band` of a half-integer."""
    out = []
    while sum(a.size for a in out) < n_want:
        x = rng.uniform(lo, hi, 4_000_000).astype(np.float32)
        v = np.abs(orc.gelu(x) * inv).astype(np.float32)
        d = np.abs(v - np.floor(v) - np.float32(0.5))
        out.append(x[d < band])
    return np.concatenate(out)[:n_want]


def test_gelu_cert_near_rounding_boundaries(gpu_lib, dev, orc):
    """Rows whose elements mostly sit within 2e-5 of a rounding boundary (inside the kernel's
    re-quantisation band), with ties exactly on .5 among them."""
    rng = np.random.default_rng(7)
    xmax = np.float32(3.0)
    m = orc.gelu(np.array([xmax], np.float32))[0]
    inv = np.float32(1.0) / (np.float32(m) / np.float32(127.0))
    pool = _near_ties(orc, rng, inv, -4.0, 2.9, 4000)
    assert pool.size == 4000
    x = np.clip(rng.standard_normal((16, K)), -4.0, 2.9).astype(np.float32)
    for r in range(x.shape[0]):
        idx = rng.choice(K, size=1500, replace=False)
        x[r, idx] = rng.choice(pool, size=1500)
        x[r, rng.integers(0, K)] = xmax
    _check(gpu_lib, dev, orc, x)


def test_gelu_cert_near_tied_maxima(gpu_lib, dev, orc):
    """The largest GELU values of a row differ by less than the approximation's error: the
    scale must come from the exact maximum."""
    rng = np.random.default_rng(8)
    x = rng.standard_normal((24, K)).astype(np.float32)
    top = np.float32(3.5)
    for r in range(x.shape[0]):
        vals = [top]
        for _ in range(1 + r % 6):
            vals.append(np.nextafter(vals[-1], np.float32(0)))
        for v in vals:
            x[r, rng.integers(0, K)] = v
        if r % 3 == 0:
            x[r, rng.integers(0, K)] = -top  # |g| of a negative input is tiny: not a candidate
    _check(gpu_lib, dev, orc, x)


def test_gelu_cert_special_rows(gpu_lib, dev, orc):
    """Rows with NaN / inf / huge values (the exact-row path), rows whose GELU vanishes or is
    tiny everywhere (every element a candidate and near a boundary), an all-zero row, rows whose
    largest |gelu| lies on the negative side or just above it, and a row count that is not a
    multiple of the block's 8 rows."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal((13, K)).astype(np.float32)
    x[0, 5] = np.nan
    x[1, 7] = np.inf
    x[2, 9] = -np.inf
    x[3, 11] = 3e38
    x[4, :] = -20.0
    x[5, :] = rng.uniform(-6.0, -4.0, K).astype(np.float32)
    x[6, :] = 0.0
    x[7, :] = rng.uniform(-1e-30, 1e-30, K).astype(np.float32)
    x[8, :] = -x[8, :] ** 2 - 3.0
    x[9, :] = rng.uniform(-2.0, 0.28, K).astype(np.float32)   # largest |gelu| on the negative side
    x[10, :] = rng.uniform(-1.0, 0.4, K).astype(np.float32)   # largest |gelu| just above 0.171
    _check(gpu_lib, dev, orc, x)
