"""GPU parity of the tcgen05 int8 GEMM through the reference ABI (wp_gemm family) against the
oracle (src/kernels.rs restated) and an int64 numpy matmul.

Bar: int32 accumulators bit-exact; fp32 epilogue bit-exact (same operation order as
src/kernels.rs:53); re-quantised int8 bit-exact for wp_gemm_q; wp_gemm_qg within one int8
step where CUDA's tanhf and glibc's tanhf differ in the last place (tolerance written below).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
NONE = 2 ** 64 - 1


def make_ctx(L, w_list):
    """Pack int8 weight matrices (and fp32 vectors) 256-byte aligned like build_plan."""
    parts, offs, size = [], [], 0
    for a in w_list:
        pad = (-size) % 256
        parts.append(b"\0" * pad)
        size += pad
        offs.append(size)
        b = np.ascontiguousarray(a).tobytes()
        parts.append(b)
        size += len(b)
    blob = np.frombuffer(b"".join(parts), np.uint8).copy()
    ctx = L.wp_create(blob.ctypes.data, blob.size)
    assert ctx
    return ctx, offs, blob


@pytest.mark.parametrize("M,K,N", [(1, 512, 512), (5, 64, 11), (127, 512, 2048), (128, 2048, 512),
                                   (129, 3840, 512), (400, 512, 2048), (390, 512, 10504), (1000, 512, 1536),
                                   (64, 48, 40), (33, 40, 24), (300, 1024, 4096)])
def test_gemm_i32_exact(gpu_lib, dev, M, K, N):
    L = gpu_lib
    rng = np.random.default_rng(M * 7 + K + N)
    a = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ctx, offs, _ = make_ctx(L, [w])
    try:
        pa = dev.put(a)
        po = dev.empty(M * N * 4)
        assert L.wp_gemm_i32(ctx, pa, M, K, offs[0], N, None, po) == 0
        assert L.wp_sync(ctx) == 0
        got = dev.get(po, (M, N), np.int32)
        ref = (a.astype(np.int64) @ w.astype(np.int64).T).astype(np.int32)
        np.testing.assert_array_equal(got, ref)
    finally:
        L.wp_destroy(ctx)


def test_gemm_extreme_values(gpu_lib, dev):
    """All +-127 / -128 operands: the largest accumulators of the model (K=3840)."""
    L = gpu_lib
    M, K, N = 130, 3840, 64
    a = np.full((M, K), 127, np.int8)
    a[1::2] = -127
    w = np.full((N, K), -128, np.int8)
    w[::3] = 127
    ctx, offs, _ = make_ctx(L, [w])
    try:
        pa, po = dev.put(a), dev.empty(M * N * 4)
        assert L.wp_gemm_i32(ctx, pa, M, K, offs[0], N, None, po) == 0
        assert L.wp_sync(ctx) == 0
        np.testing.assert_array_equal(dev.get(po, (M, N), np.int32),
                                      (a.astype(np.int64) @ w.astype(np.int64).T).astype(np.int32))
    finally:
        L.wp_destroy(ctx)


@pytest.mark.parametrize("M,K,N", [(400, 512, 2048), (17, 2048, 512), (390, 512, 10504), (3, 3840, 512)])
def test_wp_gemm_fp32_bit_exact_vs_oracle(gpu_lib, dev, orc, M, K, N):
    """Config 0 with per-tensor and per-channel scales and bias."""
    L = gpu_lib
    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N).astype(np.float32)
    b = (0.02 * rng.standard_normal(N)).astype(np.float32)
    q, s = orc.quant(x)
    ctx, offs, _ = make_ctx(L, [w, b])
    try:
        pq, ps, pws, pb = dev.put(q), dev.put(s), dev.put(ws), dev.put(b)
        po = dev.empty(M * N * 4)
        # v1: per-tensor scale, bias by blob offset (src/gpu.rs:260-264)
        assert L.wp_gemm(ctx, pq, ps, M, K, offs[0], N, 0.0123, offs[1], po) == 0
        assert L.wp_sync(ctx) == 0
        np.testing.assert_array_equal(dev.get(po, (M, N), np.float32), orc.qgemm(q, s, w, 0.0123, bias=b))
        # no bias
        assert L.wp_gemm(ctx, pq, ps, M, K, offs[0], N, 0.0123, NONE, po) == 0
        assert L.wp_sync(ctx) == 0
        np.testing.assert_array_equal(dev.get(po, (M, N), np.float32), orc.qgemm(q, s, w, 0.0123))
        # per-output-channel scale
        assert L.wp_gemm2_pc(ctx, pq, ps, M, K, offs[0], N, pws, pb, None, po) == 0
        assert L.wp_sync(ctx) == 0
        np.testing.assert_array_equal(dev.get(po, (M, N), np.float32), orc.qgemm(q, s, w, 0.0, ws_vec=ws, bias=b))
        # v2 with explicit (legacy) stream and device bias
        assert L.wp_gemm2(ctx, pq, ps, M, K, offs[0], N, 0.5, pb, None, po) == 0
        assert L.wp_sync(ctx) == 0
        np.testing.assert_array_equal(dev.get(po, (M, N), np.float32), orc.qgemm(q, s, w, 0.5, bias=b))
    finally:
        L.wp_destroy(ctx)


@pytest.mark.parametrize("N", [512, 2048, 1000])
def test_wp_gemm_q_and_qg(gpu_lib, dev, orc, N):
    L = gpu_lib
    M, K = 300, 512
    rng = np.random.default_rng(N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    b = (0.3 * rng.standard_normal(N)).astype(np.float32)
    q, s = orc.quant(x)
    ws = 1.0 / (73.6 * np.sqrt(K))
    ctx, offs, _ = make_ctx(L, [w])
    try:
        pq, ps, pb = dev.put(q), dev.put(s), dev.put(b)
        oq, osc = dev.empty(M * N), dev.empty(M * 4)
        y = orc.qgemm(q, s, w, ws, bias=b)
        assert L.wp_gemm_q(ctx, pq, ps, M, K, offs[0], N, ws, pb, None, oq, osc) == 0
        assert L.wp_sync(ctx) == 0
        rq, rs = orc.quant(y)
        np.testing.assert_array_equal(dev.get(osc, (M,), np.float32), rs)
        np.testing.assert_array_equal(dev.get(oq, (M, N), np.int8), rq)
        assert L.wp_gemm_qg(ctx, pq, ps, M, K, offs[0], N, ws, pb, None, oq, osc) == 0
        assert L.wp_sync(ctx) == 0
        gq, gs = orc.quant(orc.gelu(y))
        # the GELU epilogue evaluates the restated glibc tanhf in the reference's order: the
        # scales and int8 values are identical, not just close
        np.testing.assert_array_equal(dev.get(osc, (M,), np.float32), gs)
        np.testing.assert_array_equal(dev.get(oq, (M, N), np.int8), gq)
    finally:
        L.wp_destroy(ctx)


def test_wp_gemm_error_codes(gpu_lib, dev):
    """csrc/wtlgpu.cu:536-538,715-723: -1 args, 0 for empty shapes, -2 out-of-blob offsets."""
    L = gpu_lib
    w = np.ones((16, 64), np.int8)
    ctx, offs, blob = make_ctx(L, [w])
    try:
        pa, ps, po = dev.empty(64 * 4), dev.empty(16), dev.empty(4 * 16 * 4)
        assert L.wp_gemm(ctx, None, ps, 4, 64, 0, 16, 1.0, NONE, po) == -1
        assert L.wp_gemm(ctx, pa, None, 4, 64, 0, 16, 1.0, NONE, po) == -1
        assert L.wp_gemm(ctx, pa, ps, 4, 64, 0, 16, 1.0, NONE, None) == -1
        assert L.wp_gemm(ctx, pa, ps, 0, 64, 0, 16, 1.0, NONE, po) == 0
        assert L.wp_gemm(ctx, pa, ps, 4, 64, 0, 0, 1.0, NONE, po) == 0
        assert L.wp_gemm(ctx, pa, ps, 4, 64, blob.size, 16, 1.0, NONE, po) == -2
        assert L.wp_gemm(ctx, pa, ps, 4, 64, 0, 16, 1.0, blob.size - 8, po) == -2
        assert L.wp_gemm_q(ctx, pa, ps, 4, 64, 0, 16, 1.0, None, None, None, ps) == -1
        assert L.wp_quant_rows(po, 0, 16, None, pa, ps) == 0
        assert L.wp_devptr(ctx, blob.size + 1) is None
        assert L.wp_devptr(ctx, 0) is not None
        assert L.wp_sync(ctx) == 0
    finally:
        L.wp_destroy(ctx)


def test_capture_replay_and_stream_switch(gpu_lib, dev, orc):
    """wp_capture_begin switches the call stream to the private capturable stream for good;
    replay reproduces the eager result; errors: end without begin -12, double begin -10,
    set_stream during capture -16, empty capture -14 (csrc/wtlgpu.cu:751-847)."""
    L = gpu_lib
    M, K, N = 200, 512, 512
    rng = np.random.default_rng(1)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q, s = orc.quant(x)
    ctx, offs, _ = make_ctx(L, [w])
    try:
        pq, ps, po = dev.put(q), dev.put(s), dev.empty(M * N * 4)
        assert L.wp_stream(ctx) is None
        e = C.c_void_p()
        assert L.wp_capture_end(ctx, C.byref(e)) == -12
        assert L.wp_capture_begin(ctx) == 0
        assert L.wp_stream(ctx) is not None
        assert L.wp_is_capturing(ctx) == 1
        assert L.wp_capture_begin(ctx) == -10
        assert L.wp_set_stream(ctx, None) == -16
        assert L.wp_gemm(ctx, pq, ps, M, K, offs[0], N, 0.01, NONE, po) == 0
        assert L.wp_capture_end(ctx, C.byref(e)) == 0 and e.value
        assert L.wp_graph_count(ctx) >= 1
        zero = np.zeros((M, N), np.float32)
        assert L.wp_h2d(po, zero.ctypes.data, zero.nbytes) == 0
        assert L.wp_replay(ctx, e.value) == 0
        assert L.wp_sync(ctx) == 0
        np.testing.assert_array_equal(dev.get(po, (M, N), np.float32), orc.qgemm(q, s, w, 0.01))
        assert L.wp_graph_free(ctx, e.value) == 0
        # empty capture -> -14, stream left usable
        assert L.wp_capture_begin(ctx) == 0
        assert L.wp_capture_end(ctx, C.byref(e)) == -14 and not e.value
        assert L.wp_is_capturing(ctx) == 0
        assert L.wp_gemm(ctx, pq, ps, M, K, offs[0], N, 0.01, NONE, po) == 0
        assert L.wp_sync(ctx) == 0
    finally:
        L.wp_destroy(ctx)


def test_bounded_wait_runs_out_and_context_recovers(gpu_lib, dev):
    """Failure handling without a GPU fault: every mbarrier wait of the tcgen05 GEMM is bounded.
    wp_gemm_i32_wait_probe runs one GEMM whose producer issues no loads, with a 1 ms limit, so
    the MMA and epilogue waits run out with nothing in flight; the kernel records the cause,
    releases its tensor memory and returns.  wp_sync reports -21 once, and a normal GEMM on the
    same context afterwards is exact."""
    L = gpu_lib
    M, K, N = 256, 512, 512
    rng = np.random.default_rng(5)
    a = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ctx, offs, _ = make_ctx(L, [w])
    try:
        pa, po = dev.put(a), dev.empty(M * N * 4)
        assert L.wp_gemm_i32_wait_probe(ctx, pa, M, K, offs[0], N, None, po, 0) == -2
        assert L.wp_gemm_i32_wait_probe(ctx, pa, M, K, offs[0], N, None, po, 1_000_000) == 0
        assert L.wp_sync(ctx) == -21          # the waits ran out and said so
        assert L.wp_sync(ctx) == 0            # reported once, then cleared
        assert L.wp_gemm_i32(ctx, pa, M, K, offs[0], N, None, po) == 0
        assert L.wp_sync(ctx) == 0
        ref = (a.astype(np.int64) @ w.astype(np.int64).T).astype(np.int32)
        np.testing.assert_array_equal(dev.get(po, (M, N), np.int32), ref)
    finally:
        L.wp_destroy(ctx)
