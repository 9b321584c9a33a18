"""ctypes wrapper of liboracle.so -- TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's CPU path (see wasr_oracle.h).  Imported only by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / `--impl reference` leg, and
there only as the checker or the timed CPU baseline, never as the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "wo_set_threads": (None, [I]), "wo_get_threads": (I, []),
            "wo_quant": (None, [P, I64, I, P, P]),
            "wo_dot1": (C.c_int32, [P, P, I]),
            "wo_qgemm": (None, [P, P, I64, I, P, I, F, P, P, P]),
            "wo_qgemm_acc": (None, [P, I64, I, P, I, P]),
            "wo_dotf": (F, [P, P, I]),
            "wo_norm": (None, [P, I64, I, P, P, P]),
            "wo_gelu": (F, [F]),
            "wo_libm_tanhf": (None, [P, P, I64]), "wo_libm_expf": (None, [P, P, I64]),
            "wo_gelu_array": (None, [P, P, I64]),
            "wo_attention": (None, [P, P, P, I, P]),
            "wo_frontend": (I, [P, I, P, P, P, P]),
            "wo_conv1": (None, [P, I, P, P]),
            "wo_conv2": (None, [P, I, P, P]),
            "wo_conv3": (None, [P, I, P, P]),
            "wo_forward": (I, [P, P, P, I, P, P]),
            "wo_run_post": (I, [P, P, I, P, P, P]),
            "wo_argmax": (C.c_uint32, [P, I]),
            "wo_ctc": (I64, [P, I64, P]),
            "wo_fbank_frame": (None, [P, P]),
            "wo_fbank": (I64, [P, I64, P, I64, P]),
            "wo_transcribe": (I64, [P, P, P, I64, P, I, I, I, P, I64, P]),
            "wo_stream_commit": (I, [P, P, P, I64, P, I, I, I, P, P, P, I64, P]),
            "wo_stream_tail": (I64, [P, P, P, I64, P, I, I64, P, I64, I, P, I64, P]),
            "wo_text": (I64, [P, I64, P, I64, P, I64]),
            "wo_tidy": (I64, [C.c_char_p, I]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data if a is not None else None


def set_threads(n: int):
    lib().wo_set_threads(int(n))


def threads() -> int:
    return lib().wo_get_threads()


def quant(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    t, k = x.shape
    q = np.empty((t, k), np.int8)
    s = np.empty(t, np.float32)
    lib().wo_quant(_p(x), t, k, _p(q), _p(s))
    return q, s


def qgemm(xq, xs, w, ws, ws_vec=None, bias=None):
    xq = np.ascontiguousarray(xq, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    t, k = xq.shape
    n = w.shape[0]
    out = np.empty((t, n), np.float32)
    xs = np.ascontiguousarray(xs, np.float32)
    wv = None if ws_vec is None else np.ascontiguousarray(ws_vec, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().wo_qgemm(_p(xq), _p(xs), t, k, _p(w), n, float(ws), _p(wv), _p(b), _p(out))
    return out


def qgemm_acc(xq, w):
    xq = np.ascontiguousarray(xq, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    t, k = xq.shape
    n = w.shape[0]
    acc = np.empty((t, n), np.int32)
    lib().wo_qgemm_acc(_p(xq), t, k, _p(w), n, _p(acc))
    return acc


def dot1(a, b):
    a = np.ascontiguousarray(a, np.int8)
    b = np.ascontiguousarray(b, np.int8)
    return int(lib().wo_dot1(_p(a), _p(b), a.size))


def norm(x, g, b):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    g = np.ascontiguousarray(g, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    lib().wo_norm(_p(x), x.shape[0], x.shape[1], _p(g), _p(b), _p(y))
    return y


def _map(fn, x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    fn(_p(x), _p(y), x.size)
    return y


def gelu(x: np.ndarray) -> np.ndarray:
    """src/model.rs:710-712 (glibc tanhf)."""
    return _map(lib().wo_gelu_array, x)


def libm_tanhf(x):
    return _map(lib().wo_libm_tanhf, x)


def libm_expf(x):
    return _map(lib().wo_libm_expf, x)


def attention(q, k, v):
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    t = q.shape[0]
    out = np.empty((t, 512), np.float32)
    lib().wo_attention(_p(q), _p(k), _p(v), t, _p(out))
    return out


def frontend(x, c1, c2, c3):
    x = np.ascontiguousarray(x, np.float32)
    t = x.shape[0]
    t1 = (t - 5) // 5 + 1 if t >= 5 else 0
    y3 = np.zeros((max(t1, 1), 3840), np.float32)
    lib().wo_frontend(_p(x), t, _p(np.ascontiguousarray(c1, np.float32)),
                      _p(np.ascontiguousarray(c2, np.float32)),
                      _p(np.ascontiguousarray(c3, np.float32)), _p(y3))
    return y3[:t1]


def conv1(x, c1):
    """The conv1 stage alone (src/model.rs:398-418): x [t][40] -> y1 [t][32][40]."""
    x = np.ascontiguousarray(x, np.float32)
    t = x.shape[0]
    y1 = np.zeros((max(t, 1), 32, 40), np.float32)
    lib().wo_conv1(_p(x), t, _p(np.ascontiguousarray(c1, np.float32)), _p(y1))
    return y1[:t]


def conv2(y1, c2):
    """The conv2 stage alone (src/model.rs:420-444): y1 [t][32][40] -> y2 [t1][64][41]."""
    y1 = np.ascontiguousarray(y1, np.float32)
    t = y1.shape[0]
    t1 = (t - 5) // 5 + 1 if t >= 5 else 0
    y2 = np.zeros((max(t1, 1), 64, 41), np.float32)
    lib().wo_conv2(_p(y1), t, _p(np.ascontiguousarray(c2, np.float32)), _p(y2))
    return y2[:t1]


def conv3(y2, c3):
    """The conv3 stage alone (src/model.rs:446-468): y2 [t1][64][41] -> y3 [t1][3840]."""
    y2 = np.ascontiguousarray(y2, np.float32)
    t1 = y2.shape[0]
    y3 = np.zeros((max(t1, 1), 3840), np.float32)
    lib().wo_conv3(_p(y2), t1, _p(np.ascontiguousarray(c3, np.float32)), _p(y3))
    return y3[:t1]


def forward(blob, plan, x, want_logits=False):
    x = np.ascontiguousarray(x, np.float32)
    t = x.shape[0]
    t1 = (t - 5) // 5 + 1 if t >= 5 else 0
    ids = np.zeros(max(t1, 1), np.uint32)
    lo = np.zeros((max(t1, 1), plan.vocab), np.float32) if want_logits else None
    lib().wo_forward(_p(blob), C.byref(plan), _p(x), t, _p(ids), _p(lo))
    if want_logits:
        return ids[:t1], lo[:t1]
    return ids[:t1]


def fbank(pcm: np.ndarray):
    pcm = np.ascontiguousarray(pcm, np.int16)
    n = lib().wo_fbank(_p(pcm), pcm.size, None, 0, None)
    feats = np.zeros((max(n, 1), 40), np.float32)
    sil = np.zeros(40, np.float32)
    lib().wo_fbank(_p(pcm), pcm.size, _p(feats), n, _p(sil))
    return feats[:n], sil


def fbank_frame(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.int16)
    out = np.zeros(40, np.float64)
    lib().wo_fbank_frame(_p(x), _p(out))
    return out


def transcribe(blob, plan, feats, sil, prev=200, blk=1600, post=100):
    feats = np.ascontiguousarray(feats, np.float32)
    sil = np.ascontiguousarray(sil, np.float32)
    n = feats.shape[0]
    cap = n // 5 + 64
    ids = np.zeros(cap, np.uint32)
    nf = C.c_int(0)
    m = lib().wo_transcribe(_p(blob), C.byref(plan), _p(feats), n, _p(sil), prev, blk, post,
                            _p(ids), cap, C.byref(nf))
    assert m >= 0
    return ids[:m], nf.value


def ctc(ids):
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.zeros(max(ids.size, 1), np.uint32)
    m = lib().wo_ctc(_p(ids), ids.size, _p(out))
    return out[:m]


# ---- text output (Model::text src/model.rs:620-642, tidy src/stream.rs:203-210)
def text(ids, vocab) -> str:
    """ids -> text by the C restatement of Model::text."""
    ids = np.ascontiguousarray(ids, np.uint32)
    toks = [t.encode("utf-8") for t in vocab]
    arr = (C.c_char_p * len(toks))(*toks)
    cap = 16 + sum(len(toks[i]) + 1 for i in ids.tolist() if i < len(toks))
    out = C.create_string_buffer(cap)
    n = lib().wo_text(_p(ids), ids.size, C.cast(arr, C.c_void_p), len(toks), C.cast(out, C.c_void_p), cap)
    if n < 0:
        raise ValueError("id outside the vocabulary")
    return out.raw[:n].decode("utf-8")


def tidy(s: str, trim_end: bool = False) -> str:
    """tidy() of the C restatement; trim_end also strips trailing punctuation (partial())."""
    buf = C.create_string_buffer(s.encode("utf-8"))
    n = lib().wo_tidy(buf, 1 if trim_end else 0)
    return buf.raw[:n].decode("utf-8")


# ---- streaming schedule (src/stream.rs:58-168)
class Stream:
    """The reference's Stream restated on the oracle: the features of the audio so far come from
    the whole-prefix fbank (the rolling mean is causal, so the prefix's frames are the stream's
    frames) together with the silence frame under the prefix's final rolling mean; the commit
    loop, partial and finish ids come from the C restatement, every window through wo_forward.
    vocab None: partial() / finish() return ids; else text as Stream::partial / finish do."""

    def __init__(self, blob, plan, vocab=None, prev=200, blk=400, post=100):
        self.blob, self.plan, self.vocab = blob, plan, vocab
        self.prev, self.blk, self.post = prev, blk, post
        self.pcm = np.zeros(0, np.int16)
        self.s = C.c_int64(0)
        self.ids = np.zeros(64, np.uint32)
        self.n_ids = C.c_int64(0)
        self.n_fwd = 0
        self.feats = np.zeros((0, 40), np.float32)
        self.sil = np.zeros(40, np.float32)

    def push(self, pcm):
        self.pcm = np.concatenate([self.pcm, np.asarray(pcm, np.int16)])
        self.feats, self.sil = fbank(self.pcm)
        n = self.feats.shape[0]
        cap = n // 5 + 64
        if self.ids.size < cap:
            grown = np.zeros(cap, np.uint32)
            grown[:self.n_ids.value] = self.ids[:self.n_ids.value]
            self.ids = grown
        nf = C.c_int(0)
        rc = lib().wo_stream_commit(_p(self.blob), C.byref(self.plan), _p(self.feats), n, _p(self.sil), self.prev,
                                    self.blk, self.post, C.byref(self.s), _p(self.ids), C.byref(self.n_ids),
                                    self.ids.size, C.byref(nf))
        assert rc == 0
        self.n_fwd += nf.value

    def _tail(self, finish: bool):
        n = self.feats.shape[0]
        cap = n // 5 + 64 + self.n_ids.value
        out = np.zeros(cap, np.uint32)
        nf = C.c_int(0)
        m = lib().wo_stream_tail(_p(self.blob), C.byref(self.plan), _p(self.feats), n, _p(self.sil), self.prev,
                                 self.s.value, _p(self.ids), self.n_ids.value, 1 if finish else 0, _p(out), cap,
                                 C.byref(nf))
        assert m >= 0
        self.n_fwd += nf.value
        return out[:m]

    def partial(self):
        ids = self._tail(False)
        return ids if self.vocab is None else tidy(text(ids, self.vocab), trim_end=True)

    def finish(self):
        ids = self._tail(True)
        return ids if self.vocab is None else tidy(text(ids, self.vocab))
