"""The reference's model directory: a `.xnet` container plus `dict.decoder.utf8.txt`.

* `parse(data)` restates the container parser of src/xnet.rs:45-107: after the "XNET" magic,
  find the first offset where a complete record chain parses up to the end of the file.  A record
  is: u32 name length (1..256), name, u32 dtype, u32 quant flag, 3 x u32, u32 scale count (<= 4096),
  u32, the scales (f32), u32 zero-point bytes + those bytes, u32 rank (<= 8), the dims (u32 each),
  u32 byte length (= product of dims x element size), the data.  A zero name length ends the
  chain; at most 16 zero bytes may follow, and more than 100 records must have been read.
* `load_plan(dir)` restates build_plan (src/model.rs:209-237) and the vocabulary check of
  Model::load (src/model.rs:240-272): the tensors are packed into one 256-byte-aligned blob in
  build_plan's order and described by a WasrPlan, so the engine loads the reference's model files.
* `write_model_dir(dir, blob, plan)` writes a synthetic model directory that the reference's
  own loader accepts (the names, dtypes, dims and quant scales it asks for, 40 layers), with a
  dictionary of placeholder tokens; `load_plan` of that directory gives back the same blob.
"""
from __future__ import annotations

import os
import struct

import numpy as np

from .abi import C1, C2, C3, D, FF, FLAT, MAX_LAYERS, WASR_NONE, WasrPlan

F32, I8 = 11, 6
LAYERS = 40                       # src/model.rs: the loader requires all 40 encoder layers
_ELEM = {I8: 1, 2: 1, 3: 1, 4: 2, 5: 2, 1: 4, 7: 4, 8: 4, F32: 4, 9: 8, 10: 8, 12: 8}


class Rec:
    __slots__ = ("dtype", "scale", "dims", "off", "len")

    def __init__(self, dtype, scale, dims, off, ln):
        self.dtype, self.scale, self.dims, self.off, self.len = dtype, scale, dims, off, ln


def _chain(d: bytes, p: int):
    out = {}
    n_all = len(d)

    def u32():
        nonlocal p
        if p + 4 > n_all:
            raise IndexError
        v = struct.unpack_from("<I", d, p)[0]
        p += 4
        return v

    def take(n):
        nonlocal p
        if n < 0 or p + n > n_all:
            raise IndexError
        b = d[p:p + n]
        p += n
        return b

    try:
        while True:
            n = u32()
            if n == 0:
                rest = d[p:]
                return out if (len(rest) <= 16 and not any(rest) and len(out) > 100) else None
            if n > 256:
                return None
            name = take(n).decode("utf-8")
            dtype = u32()
            es = _ELEM.get(dtype)
            if es is None:
                return None
            quant = u32()
            for _ in range(3):
                u32()
            ns = u32()
            u32()
            if ns > 4096:
                return None
            sc = take(ns * 4)
            scale = struct.unpack_from("<f", sc, 0)[0] if (quant != 0 and ns > 0) else None
            nz = u32()
            take(nz)
            nd = u32()
            if nd > 8:
                return None
            dims = [u32() for _ in range(nd)]
            ln = u32()
            if ln != int(np.prod(dims, dtype=np.int64)) * es:
                return None
            off = p
            take(ln)
            out[name] = Rec(dtype, scale, dims, off, ln)
    except (IndexError, UnicodeDecodeError):
        return None


def parse(d: bytes) -> dict:
    """Record table of a .xnet file (src/xnet.rs:86-107); raises ValueError when there is none."""
    if d[:4] != b"XNET":
        raise ValueError("not an xnet model file")
    p = 8
    while True:
        at = -1
        for i in range(p, len(d) - 3):   # next u32 in 1..128 followed by three zero bytes
            if 1 <= d[i] <= 128 and d[i + 1] == 0 and d[i + 2] == 0 and d[i + 3] == 0:
                at = i
                break
        if at < 0:
            raise ValueError("no xnet weight table found")
        n = d[at]
        name = d[at + 4:at + 4 + n]
        if len(name) == n and all(0x21 <= b <= 0x7E for b in name):
            m = _chain(d, at)
            if m is not None:
                return m
        p = at + 1


# ---------------------------------------------------------------- writing
def _record(name: str, dtype: int, arr: np.ndarray, scale: float | None) -> bytes:
    nb = name.encode("utf-8")
    dims = list(arr.shape)
    data = np.ascontiguousarray(arr).tobytes()
    out = [struct.pack("<I", len(nb)), nb, struct.pack("<II", dtype, 1 if scale is not None else 0),
           struct.pack("<III", 0, 0, 0)]
    if scale is not None:
        out += [struct.pack("<II", 1, 0), struct.pack("<f", scale)]
    else:
        out += [struct.pack("<II", 0, 0)]
    out += [struct.pack("<I", 0), struct.pack("<I", len(dims)), struct.pack(f"<{len(dims)}I", *dims),
            struct.pack("<I", len(data)), data]
    return b"".join(out)


def tensors_from_blob(blob: np.ndarray, plan: WasrPlan) -> list[tuple[str, int, np.ndarray, float | None]]:
    """The named tensors of a blob laid out by build_plan (synth.make_model), in the reference's
    names (src/model.rs:213-234)."""
    if plan.n_layers != LAYERS:
        raise ValueError(f"the reference loader needs {LAYERS} layers, plan has {plan.n_layers}")
    b = np.asarray(blob, np.uint8)
    vocab = plan.vocab

    def f32(off, shape):
        n = int(np.prod(shape))
        return b[off:off + 4 * n].view(np.float32).reshape(shape).copy()

    def q(m, rows=None):
        rows = m.n if rows is None else rows
        if m.scale_off != WASR_NONE:
            raise ValueError("per-channel scales have no .xnet form (the reference stores one scale per tensor)")
        return b[m.off:m.off + rows * m.k].view(np.int8).reshape(rows, m.k).copy(), float(np.float32(m.s))

    out = []
    for i in range(LAYERS):
        L = plan.layers[i]
        p = f"layers.{i}."
        for nm, off in (("prior_norm.weight", L.pn_g), ("prior_norm.bias", L.pn_b),
                        ("middle_norm.weight", L.mn_g), ("middle_norm.bias", L.mn_b)):
            out.append((p + nm, F32, f32(off, (D,)), None))
        for nm, m in (("attention.q_conv", L.q), ("attention.k_conv", L.k), ("attention.v_conv", L.v),
                      ("attention.output_transform_conv", L.o), ("feed_forward.filter_conv", L.f1),
                      ("feed_forward.output_conv", L.f2)):
            w, s = q(m)
            out.append((p + nm + ".weight_quantized_s8", I8, w, s))
        if any(getattr(L, x) != WASR_NONE for x in ("qb", "kb", "vb", "ob")):
            raise ValueError("q/k/v/o biases have no place in the reference's loader")
        out.append((p + "feed_forward.filter_conv.bias", F32, f32(L.f1b, (FF,)), None))
        out.append((p + "feed_forward.output_conv.bias", F32, f32(L.f2b, (D,)), None))
    w, s = q(plan.lin)
    out.append(("frontend.linear.weight_quantized_s8", I8, w, s))
    out.append(("frontend.linear.bias", F32, f32(plan.lin_b, (D,)), None))
    w, s = q(plan.out, rows=vocab)   # the padding rows are build_plan's, not the file's
    out.append(("output_conv.weight_quantized_s8", I8, w, s))
    out.append(("output_conv.bias", F32, f32(plan.out_b, (vocab,)), None))
    out.append(("frontend.conv2d.weight", F32, f32(plan.c1, (C1, 1, 5, 5)), None))
    out.append(("frontend.conv2d_1.weight", F32, f32(plan.c2, (C2, C1, 7, 7)), None))
    out.append(("frontend.conv2d_2.weight", F32, f32(plan.c3, (C3, C2, 3, 3)), None))
    return out


def rust_lines(s: str) -> list[str]:
    """Rust's str::lines: split at '\\n', one trailing '\\r' removed per line, and no empty last
    line for a final line ending (other Unicode line separators stay inside the line)."""
    if not s:
        return []
    parts = s.split("\n")
    if s.endswith("\n"):
        parts.pop()
    return [p[:-1] if p.endswith("\r") else p for p in parts]


def read_vocab(path: str) -> list[str]:
    """dict.decoder.utf8.txt as Model::load reads it (src/model.rs:267-271): UTF-8 (invalid
    bytes are an error), lines as str::lines gives them, the token the second space-separated
    field ("" when there is none)."""
    with open(path, "rb") as f:
        data = f.read().decode("utf-8")
    out = []
    for ln in rust_lines(data):
        fields = ln.split(" ")
        out.append(fields[1] if len(fields) > 1 else "")
    return out


def write_model_dir(path: str, blob: np.ndarray, plan: WasrPlan, tokens: list[str] | None = None) -> None:
    """Write `model.xnet` and `dict.decoder.utf8.txt` for a 40-layer blob/plan into `path`."""
    os.makedirs(path, exist_ok=True)
    recs = tensors_from_blob(blob, plan)
    with open(os.path.join(path, "model.xnet"), "wb") as f:
        f.write(b"XNET" + struct.pack("<I", 1))
        for name, dtype, arr, scale in recs:
            f.write(_record(name, dtype, arr, scale))
        f.write(struct.pack("<I", 0) + bytes(12))
    toks = tokens if tokens is not None else [f"t{i}" for i in range(plan.vocab)]
    if len(toks) != plan.vocab:
        raise ValueError("one token per output id")
    with open(os.path.join(path, "dict.decoder.utf8.txt"), "w", encoding="utf-8") as f:
        for i, t in enumerate(toks):
            f.write(f"{i} {t}\n")


# ---------------------------------------------------------------- loading (build_plan)
class _Blob:
    def __init__(self):
        self.parts, self.size = [], 0

    def add(self, raw: bytes) -> int:
        pad = (-self.size) % 256
        if pad:
            self.parts.append(b"\0" * pad)
            self.size += pad
        off = self.size
        self.parts.append(raw)
        self.size += len(raw)
        return off

    def bytes(self) -> np.ndarray:
        return np.frombuffer(b"".join(self.parts), np.uint8).copy()


def load_plan(path: str):
    """(blob, WasrPlan, tokens) from a model directory, as build_plan packs it."""
    xs = sorted(f for f in os.listdir(path) if f.endswith(".xnet"))
    if not xs:
        raise FileNotFoundError("no .xnet file in the model directory")
    with open(os.path.join(path, xs[0]), "rb") as f:
        d = f.read()
    r = parse(d)

    def rec(name):
        if name not in r:
            raise KeyError(f"model lacks {name}")
        return r[name]

    def f32(name, dims):
        x = rec(name)
        if x.dtype != F32 or x.dims != list(dims):
            raise ValueError(f"{name} shape {x.dims}")
        return d[x.off:x.off + x.len]

    def qrec(name, n, k):
        x = rec(name + ".weight_quantized_s8")
        if x.dtype != I8 or len(x.dims) < 2 or x.dims[:2] != [n, k] or x.len != n * k:
            raise ValueError(f"{name} shape {x.dims}")
        if x.scale is None:
            raise ValueError(f"{name} lacks its quantisation scale")
        return x

    vocab = rec("output_conv.bias").dims[0] if rec("output_conv.bias").dims else 0
    tokens = read_vocab(os.path.join(path, "dict.decoder.utf8.txt"))
    if len(tokens) != vocab:
        raise ValueError(f"vocabulary size {len(tokens)} != model output {vocab}")
    out_n = (vocab + 3) // 4 * 4
    b = _Blob()
    plan = WasrPlan()
    plan.n_layers, plan.vocab, plan.out_n = LAYERS, vocab, out_n

    def mat(m, name, n, k, pad=0):
        x = qrec(name, n, k)
        raw = d[x.off:x.off + x.len]
        m.off = b.add(raw if pad == 0 else raw + bytes(pad * k))
        m.s, m.n, m.k, m.scale_off = x.scale, n + pad, k, WASR_NONE

    for i in range(LAYERS):
        L = plan.layers[i]
        p = f"layers.{i}."
        L.pn_g = b.add(f32(p + "prior_norm.weight", [D]))
        L.pn_b = b.add(f32(p + "prior_norm.bias", [D]))
        L.mn_g = b.add(f32(p + "middle_norm.weight", [D]))
        L.mn_b = b.add(f32(p + "middle_norm.bias", [D]))
        mat(L.q, p + "attention.q_conv", D, D)
        mat(L.k, p + "attention.k_conv", D, D)
        mat(L.v, p + "attention.v_conv", D, D)
        mat(L.o, p + "attention.output_transform_conv", D, D)
        mat(L.f1, p + "feed_forward.filter_conv", FF, D)
        L.f1b = b.add(f32(p + "feed_forward.filter_conv.bias", [FF]))
        mat(L.f2, p + "feed_forward.output_conv", D, FF)
        L.f2b = b.add(f32(p + "feed_forward.output_conv.bias", [D]))
        L.qb = L.kb = L.vb = L.ob = WASR_NONE
    mat(plan.lin, "frontend.linear", D, FLAT)
    plan.lin_b = b.add(f32("frontend.linear.bias", [D]))
    mat(plan.out, "output_conv", vocab, D, pad=out_n - vocab)
    ob = f32("output_conv.bias", [vocab]) + np.full(out_n - vocab, -1e30, np.float32).tobytes()
    plan.out_b = b.add(ob)
    plan.c1 = b.add(f32("frontend.conv2d.weight", [C1, 1, 5, 5]))
    plan.c2 = b.add(f32("frontend.conv2d_1.weight", [C2, C1, 7, 7]))
    plan.c3 = b.add(f32("frontend.conv2d_2.weight", [C3, C2, 3, 3]))
    assert LAYERS <= MAX_LAYERS
    return b.bytes(), plan, tokens
