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
            "wo_forward": (I, [P, P, P, I, P, P]),
            "wo_run_post": (I, [P, P, I, P, P, P]),
            "wo_argmax": (C.c_uint32, [P, I]),
            "wo_ctc": (I64, [P, I64, P]),
            "wo_fbank_frame": (None, [P, P]),
            "wo_fbank": (I64, [P, I64, P, I64, P]),
            "wo_transcribe": (I64, [P, P, P, I64, P, I, I, I, P, I64, P]),
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
