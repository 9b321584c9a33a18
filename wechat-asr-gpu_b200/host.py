"""Host side over libwasr_gpu.so.

``Engine``      the additive batched engine (include/wasr.h): stacked ragged windows,
                batch transcription with the reference stream schedule, host fbank.
``Gpu``         mirror of the reference's Rust FFI wrapper ``Gpu`` (src/gpu.rs:97-311): device
                activation buffers sized for TMAX and one thin method per ABI call, with the
                same names and argument meaning.
``WindowModel`` mirror of ``Model::run_gpu`` / ``window_ops`` / ``warm_shapes``
                (src/model.rs:504-619): one window per forward through the reference ABI,
                CUDA graphs keyed by t1.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import abi
from .abi import D, DIM, FF, FLAT, HEADS, WASR_F_DEVICE, WASR_F_NOSYNC, WASR_NONE, ptr

NO_BIAS = (1 << 64) - 1  # src/gpu.rs:88
TMAX = 512               # src/model.rs:35


def _lib():
    return abi.load()


def fbank(pcm: np.ndarray):
    """Host fbank of the product (src/fbank.rs): returns (feats [n][40] f32, silence [40])."""
    pcm = np.ascontiguousarray(pcm, np.int16)
    L = _lib()
    n = L.wasr_fbank(ptr(pcm), pcm.size, None, 0, None)
    feats = np.zeros((max(n, 1), DIM), np.float32)
    sil = np.zeros(DIM, np.float32)
    rc = L.wasr_fbank(ptr(pcm), pcm.size, ptr(feats), n, ptr(sil))
    if rc < 0:
        raise RuntimeError(f"wasr_fbank rc={rc}")
    return feats[:n], sil


def ctc_collapse(ids) -> np.ndarray:
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.zeros(max(ids.size, 1), np.uint32)
    k = _lib().wasr_ctc_collapse(ptr(ids), ids.size, ptr(out))
    return out[:k]


class Engine:
    """Batched engine on one device (include/wasr.h)."""

    def __init__(self, blob: np.ndarray, plan: abi.WasrPlan, device: int = 0, max_rows: int = 16384):
        self.L = _lib()
        self.blob = np.ascontiguousarray(blob, np.uint8)
        self.plan = plan
        self.m = self.L.wasr_model_create(ptr(self.blob), self.blob.size, C.byref(plan), device, max_rows)
        if not self.m:
            raise RuntimeError("wasr_model_create failed")
        self.device = device

    @classmethod
    def from_model_dir(cls, path: str, device: int = 0, max_rows: int = 16384) -> "Engine":
        """Engine over the reference's model directory (.xnet + dict.decoder.utf8.txt), packed
        the way build_plan packs it (src/model.rs:209-237); the vocabulary is kept as `tokens`."""
        from . import xnet
        blob, plan, tokens = xnet.load_plan(path)
        eng = cls(blob, plan, device=device, max_rows=max_rows)
        eng.tokens = tokens
        return eng

    def close(self):
        if self.m:
            self.L.wasr_model_destroy(self.m)
            self.m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr: int | None):
        return self.L.wasr_model_set_stream(self.m, stream_ptr)

    @property
    def stream(self) -> int:
        return self.L.wasr_model_stream(self.m) or 0

    def set_graphs(self, on: bool):
        return self.L.wasr_model_set_graphs(self.m, 1 if on else 0)

    def forward(self, windows, want_logits: bool = False):
        """Host windows (list of [t][40] arrays) -> list of id arrays (and logits)."""
        t = np.array([w.shape[0] for w in windows], np.int32)
        feats = np.ascontiguousarray(np.concatenate(windows, 0) if len(windows) else np.zeros((0, DIM)),
                                     np.float32)
        t1 = np.where(t >= 5, (t - 5) // 5 + 1, 0)
        rows = int(t1.sum())
        ids = np.zeros(max(rows, 1), np.uint32)
        lo = np.zeros((max(rows, 1), self.plan.out_n), np.float32) if want_logits else None
        rc = self.L.wasr_forward(self.m, ptr(feats), ptr(t), len(windows), ptr(ids),
                                 ptr(lo) if lo is not None else None, 0)
        if rc:
            raise RuntimeError(f"wasr_forward rc={rc}")
        offs = np.concatenate([[0], np.cumsum(t1)])
        out = [ids[offs[i]:offs[i + 1]] for i in range(len(windows))]
        if want_logits:
            return out, [lo[offs[i]:offs[i + 1], :self.plan.vocab] for i in range(len(windows))]
        return out

    def forward_device(self, feats_dev: int, t: np.ndarray, ids_dev: int, sync: bool = True):
        """Device-resident forward: feats_dev / ids_dev are device addresses."""
        t = np.ascontiguousarray(t, np.int32)
        flags = WASR_F_DEVICE | (0 if sync else WASR_F_NOSYNC)
        rc = self.L.wasr_forward(self.m, feats_dev, ptr(t), t.size, ids_dev, None, flags)
        if rc:
            raise RuntimeError(f"wasr_forward rc={rc}")

    def transcribe(self, feats_list, sils, prev=200, blk=1600, post=100, feats_cat=None):
        """Per-utterance features -> per-utterance raw ids (before CTC collapse)."""
        n = np.array([f.shape[0] for f in feats_list], np.int64)
        if feats_cat is None:
            feats_cat = np.ascontiguousarray(np.concatenate(feats_list, 0), np.float32)
        sil = np.ascontiguousarray(np.stack(sils, 0), np.float32)
        cap = int(n.sum() // 5 + 64 * len(feats_list) + 64)
        ids = np.zeros(cap, np.uint32)
        off = np.zeros(len(feats_list) + 1, np.int64)
        rc = self.L.wasr_transcribe(self.m, ptr(feats_cat), ptr(n), ptr(sil), len(feats_list), prev, blk, post,
                                    ptr(ids), ptr(off), cap)
        if rc:
            raise RuntimeError(f"wasr_transcribe rc={rc}")
        return [ids[off[i]:off[i + 1]].copy() for i in range(len(feats_list))]

    def transcribe_device(self, feats_dev: int, n_frames, sil_dev: int, prev=200, blk=1600, post=100):
        """transcribe() on device-resident features (e.g. wasr_fbank_device's output): feats_dev
        holds the utterances' [frames][40] fp32 rows back to back, sil_dev their [n][40] silence
        frames (device addresses on this engine's device).  Returns per-utterance raw ids."""
        n = np.ascontiguousarray(n_frames, np.int64)
        cap = int(n.sum() // 5 + 64 * n.size + 64)
        ids = np.zeros(cap, np.uint32)
        off = np.zeros(n.size + 1, np.int64)
        rc = self.L.wasr_transcribe_device(self.m, feats_dev, ptr(n), sil_dev, n.size, prev, blk, post, ptr(ids),
                                           ptr(off), cap)
        if rc:
            raise RuntimeError(f"wasr_transcribe_device rc={rc}")
        return [ids[off[i]:off[i + 1]].copy() for i in range(n.size)]

    def error(self) -> int:
        return self.L.wasr_model_error(self.m)

    def set_profile(self, on: bool):
        return self.L.wasr_model_set_profile(self.m, 1 if on else 0)

    def profile(self):
        """Per kernel class (abi.KERNEL_CLASSES): (ms of the last execution, launches)."""
        n = len(abi.KERNEL_CLASSES)
        ms = np.zeros(n, np.float64)
        cnt = np.zeros(n, np.int64)
        rc = self.L.wasr_model_profile(self.m, ptr(ms), ptr(cnt), n)
        if rc:
            raise RuntimeError(f"wasr_model_profile rc={rc}")
        return ms, cnt

    def kernel_launches(self) -> int:
        return int(self.L.wasr_model_kernel_launches(self.m))


class Gpu:
    """Mirror of src/gpu.rs ``Gpu``: one WpCtx plus activation buffers sized for tmax."""

    def __init__(self, blob: np.ndarray, tmax: int, d: int, ff: int, vocab: int, flat: int, heads: int):
        L = self.L = _lib()
        self.blob = np.ascontiguousarray(blob, np.uint8)
        self.ctx = L.wp_create(ptr(self.blob), self.blob.size)
        if not self.ctx:
            raise RuntimeError("wp_create failed")
        self.graphs: dict[int, int] = {}
        self.tmax, self.vocab = tmax, vocab
        self.tmax_feat = 5 * (tmax - 1) + 5
        self._bufs = []

        def alloc(n):
            p = L.wp_alloc(max(n, 1))
            if not p:
                raise RuntimeError("wp_alloc failed")
            self._bufs.append(p)
            return p
        tf = self.tmax_feat
        self.x = alloc(tf * DIM * 4)
        self.y1 = alloc(tf * 32 * DIM * 4)
        self.y2 = alloc(tmax * 64 * 41 * 4)
        self.y3 = alloc(tmax * flat * 4)
        self.y3q = alloc(tmax * flat)
        self.ys = alloc(tmax * 4)
        self.h = alloc(tmax * d * 4)
        self.xq = alloc(tmax * d)
        self.xs = alloc(tmax * 4)
        self.q = alloc(tmax * d * 4)
        self.k = alloc(tmax * d * 4)
        self.v = alloc(tmax * d * 4)
        self.att = alloc(tmax * d * 4)
        self.scores = alloc(heads * tmax * tmax * 4)
        self.o = alloc(tmax * d * 4)
        self.aq = alloc(tmax * max(ff, d))
        self.asc = alloc(tmax * 4)
        self.f = alloc(tmax * ff * 4)
        self.fq = alloc(tmax * ff)
        self.fsc = alloc(tmax * 4)
        self.lo = alloc(tmax * vocab * 4)
        self.ids = alloc(tmax * 4)

    def close(self):
        if self.ctx:
            for e in self.graphs.values():
                self.L.wp_graph_free(self.ctx, e)
            for p in self._bufs:
                self.L.wp_free(p)
            self.L.wp_destroy(self.ctx)
            self.ctx = None

    def stream(self):
        return self.L.wp_stream(self.ctx)

    def capture_begin(self) -> bool:
        return self.L.wp_capture_begin(self.ctx) == 0

    def capture_end(self):
        e = C.c_void_p()
        rc = self.L.wp_capture_end(self.ctx, C.byref(e))
        return e.value if rc == 0 and e.value else None

    def replay(self, e):
        rc = self.L.wp_replay(self.ctx, e)
        assert rc == 0, f"wp_replay rc={rc}"

    def dev(self, off):
        return self.L.wp_devptr(self.ctx, off)

    def sync(self):
        rc = self.L.wp_sync(self.ctx)
        assert rc == 0, f"wp_sync rc={rc}"

    def upload_feats(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        assert self.L.wp_h2d(self.x, ptr(x), x.nbytes) == 0

    def download_ids(self, t1: int) -> np.ndarray:
        out = np.zeros(t1, np.uint32)
        assert self.L.wp_d2h(ptr(out), self.ids, t1 * 4) == 0
        return out

    def front(self, t, t1, c1, c2, c3):
        self.L.wk_front(self.stream(), self.x, self.dev(c1), self.dev(c2), self.dev(c3), t, t1, self.y1, self.y2,
                        self.y3)

    def quant_y3(self, t1):
        self.L.wk_quant(self.stream(), self.y3, t1, FLAT, self.y3q, self.ys)

    def gemm(self, xq, xs, t, k, w, n, ws, bias, out):
        rc = self.L.wp_gemm(self.ctx, xq, xs, t, k, w, n, ws, NO_BIAS if bias == WASR_NONE else bias, out)
        assert rc == 0, f"wp_gemm rc={rc} (t={t} k={k} n={n})"

    def norm_quant(self, t, d, g, b, xq, xs):
        self.L.wk_norm_quant(self.stream(), self.h, self.dev(g), self.dev(b), t, d, xq, xs)

    def add_norm_quant(self, t, d, g, b, xq, xs):
        self.L.wk_add_norm_quant(self.stream(), self.h, self.o, self.dev(g), self.dev(b), t, d, xq, xs)

    def quant(self, x, t, k, xq, xs):
        self.L.wk_quant(self.stream(), x, t, k, xq, xs)

    def gelu_quant(self, t, k, xq, xs):
        self.L.wk_gelu_quant(self.stream(), self.f, t, k, xq, xs)

    def attention(self, t, d, heads, q, k, v, out):
        rc = self.L.wk_attention_fast(self.stream(), q, k, v, t, d, heads, self.scores, out)
        assert rc == 0, f"wk_attention_fast rc={rc} (t={t})"

    def add(self, h, a, t, d):
        self.L.wk_add(self.stream(), h, a, t, d)

    def argmax(self, x, t, n, out):
        self.L.wk_argmax(self.stream(), x, t, n, out)


class WindowModel:
    """Mirror of the reference's per-window GPU forward (src/model.rs:504-619) driven through
    the reference ABI only.  The reference model has no q/k/v/o biases; a plan that has them
    is rejected here (the batched Engine supports them)."""

    def __init__(self, blob, plan: abi.WasrPlan, graphs: bool = True):
        for i in range(plan.n_layers):
            L = plan.layers[i]
            if any(b != WASR_NONE for b in (L.qb, L.kb, L.vb, L.ob)):
                raise ValueError("WindowModel follows window_ops: no q/k/v/o biases")
        self.pl = plan
        self.g = Gpu(blob, TMAX, D, FF, plan.out_n, FLAT, HEADS)
        self.graph_on = graphs

    def close(self):
        self.g.close()

    def warm_shapes(self, t1):  # src/model.rs:504-518 (nothing to warm here; kept for parity)
        return None

    def window_ops(self, t1):  # src/model.rs:520-541
        g, pl = self.g, self.pl
        g.gemm(g.y3q, g.ys, t1, FLAT, pl.lin.off, D, pl.lin.s, pl.lin_b, g.h)
        for i in range(pl.n_layers):
            l = pl.layers[i]
            g.norm_quant(t1, D, l.pn_g, l.pn_b, g.xq, g.xs)
            g.gemm(g.xq, g.xs, t1, D, l.q.off, D, l.q.s, NO_BIAS, g.q)
            g.gemm(g.xq, g.xs, t1, D, l.k.off, D, l.k.s, NO_BIAS, g.k)
            g.gemm(g.xq, g.xs, t1, D, l.v.off, D, l.v.s, NO_BIAS, g.v)
            g.attention(t1, D, HEADS, g.q, g.k, g.v, g.att)
            g.quant(g.att, t1, D, g.aq, g.asc)
            g.gemm(g.aq, g.asc, t1, D, l.o.off, D, l.o.s, NO_BIAS, g.o)
            g.add_norm_quant(t1, D, l.mn_g, l.mn_b, g.xq, g.xs)
            g.gemm(g.xq, g.xs, t1, D, l.f1.off, FF, l.f1.s, l.f1b, g.f)
            g.gelu_quant(t1, FF, g.fq, g.fsc)
            g.gemm(g.fq, g.fsc, t1, FF, l.f2.off, D, l.f2.s, l.f2b, g.o)
            g.add(g.h, g.o, t1, D)
        g.quant(g.h, t1, D, g.aq, g.asc)
        g.gemm(g.aq, g.asc, t1, D, pl.out.off, pl.out_n, pl.out.s, pl.out_b, g.lo)
        g.argmax(g.lo, t1, pl.out_n, g.ids)

    def forward(self, x: np.ndarray) -> np.ndarray:  # run_gpu, src/model.rs:546-619
        t = x.shape[0]
        if t < 5:
            return np.zeros(0, np.uint32)
        t1 = (t - 5) // 5 + 1
        g, pl = self.g, self.pl
        if t1 > g.tmax:
            raise ValueError("t1 > TMAX: the reference falls back to its CPU path here")
        g.upload_feats(x)
        g.front(t, t1, pl.c1, pl.c2, pl.c3)
        g.quant_y3(t1)
        e = g.graphs.get(t1)
        if e is not None:
            g.replay(e)
        else:
            done = False
            if self.graph_on:
                self.warm_shapes(t1)
                if g.capture_begin():
                    self.window_ops(t1)
                    e = g.capture_end()
                    if e is not None:
                        g.graphs[t1] = e
                        g.replay(e)
                        done = True
            if not done:
                self.window_ops(t1)
        g.sync()
        return g.download_ids(t1)
