"""Seeded synthetic inputs for the workloads the benchmark and tests run.

The reference's model weights (.xnet), vocabulary and audio are not public, so every input
is generated here from a seed:
  * ``make_model`` packs random-init weights into one blob in the layout the reference's
    ``build_plan`` produces (src/model.rs:148-237): every tensor 256-byte aligned, per layer
    pn_g, pn_b, mn_g, mn_b, q, k, v, o, f1, f1b, f2, f2b, then lin, lin_b, out (rows padded
    with zeros to a multiple of 4), out_b (padded with -1e30), conv1/2/3 weights.  Shapes
    follow the asserts of src/model.rs:209-234,295-302.  int8 weights are uniform in
    [-127, 127]; per-tensor scales are chosen so activations stay O(1) through 40 layers.
  * ``make_audio`` builds 16 kHz int16 audio from 5 sinusoids (80-4000 Hz, amplitudes
    U(0.05, 0.3)) plus N(0, 0.02^2) noise, peak-scaled into the int16 range.
  * ``config_lengths`` gives the utterance lengths of the benchmark configurations.
"""
from __future__ import annotations

import numpy as np

from .abi import (C1, C2, C3, D, FF, FLAT, MAX_LAYERS, WASR_NONE, WasrPlan)

VOCAB = 10502
SR = 16000


class _Blob:
    def __init__(self):
        self.parts: list[bytes] = []
        self.size = 0

    def add(self, a: np.ndarray) -> int:
        pad = (-self.size) % 256
        if pad:
            self.parts.append(b"\0" * pad)
            self.size += pad
        off = self.size
        b = np.ascontiguousarray(a).tobytes()
        self.parts.append(b)
        self.size += len(b)
        return off

    def bytes(self) -> np.ndarray:
        return np.frombuffer(b"".join(self.parts), dtype=np.uint8).copy()


def _i8(rng, n, k):
    return rng.integers(-127, 128, size=(n, k), dtype=np.int8)


def _scale(rng, k, gain=1.0):
    # uniform int8 in [-127,127] has std 73.6; keep (xq*xs)@(w*ws) at O(gain)
    return float(gain * rng.uniform(0.5, 1.0) / (73.6 * np.sqrt(k)))


def make_model(seed: int = 1, n_layers: int = 40, vocab: int = VOCAB, per_channel: bool = False,
               proj_bias: bool = False, ln_identity: bool = False):
    """Random-init model.  Returns (blob uint8 array, WasrPlan).

    per_channel: also store an fp32 per-output-channel scale vector for every matrix
        (BASELINE config 0/1 extension); the plan then points at it.
    proj_bias: add biases to the q/k/v/o projections (config 1: "bias on every projection").
    ln_identity: LayerNorm gamma = 1, beta = 0 (config 1).
    """
    assert 1 <= n_layers <= MAX_LAYERS
    rng = np.random.default_rng(seed)
    b = _Blob()
    plan = WasrPlan()
    plan.n_layers = n_layers
    plan.vocab = vocab
    out_n = (vocab + 3) // 4 * 4
    plan.out_n = out_n

    def mat(m, n, k, gain=1.0, pad_rows=0):
        w = _i8(rng, n, k)
        if pad_rows:
            w = np.concatenate([w, np.zeros((pad_rows, k), np.int8)], 0)
        m.off = b.add(w)
        m.s = _scale(rng, k, gain)
        m.n = n + pad_rows
        m.k = k
        m.scale_off = WASR_NONE
        if per_channel:
            sv = (m.s * rng.uniform(0.5, 1.5, size=n + pad_rows)).astype(np.float32)
            m.scale_off = b.add(sv)

    def vec(n, std, mean=0.0):
        return b.add((mean + std * rng.standard_normal(n)).astype(np.float32))

    for i in range(n_layers):
        L = plan.layers[i]
        if ln_identity:
            L.pn_g = b.add(np.ones(D, np.float32)); L.pn_b = b.add(np.zeros(D, np.float32))
            L.mn_g = b.add(np.ones(D, np.float32)); L.mn_b = b.add(np.zeros(D, np.float32))
        else:
            L.pn_g = vec(D, 0.1, 1.0); L.pn_b = vec(D, 0.05)
            L.mn_g = vec(D, 0.1, 1.0); L.mn_b = vec(D, 0.05)
        mat(L.q, D, D, 1.0)
        mat(L.k, D, D, 1.0)
        mat(L.v, D, D, 1.0)
        mat(L.o, D, D, 0.7)
        mat(L.f1, FF, D, 1.0)
        L.f1b = vec(FF, 0.02)
        mat(L.f2, D, FF, 1.2)
        L.f2b = vec(D, 0.02)
        if proj_bias:
            L.qb, L.kb, L.vb, L.ob = vec(D, 0.02), vec(D, 0.02), vec(D, 0.02), vec(D, 0.02)
        else:
            L.qb = L.kb = L.vb = L.ob = WASR_NONE
    mat(plan.lin, D, FLAT, 3.0)
    plan.lin_b = vec(D, 0.02)
    mat(plan.out, vocab, D, 4.0, pad_rows=out_n - vocab)
    ob = np.concatenate([(0.02 * rng.standard_normal(vocab)).astype(np.float32),
                         np.full(out_n - vocab, -1e30, np.float32)])
    plan.out_b = b.add(ob)
    plan.c1 = b.add((rng.standard_normal((C1, 1, 5, 5)) * np.sqrt(2.0 / 25)).astype(np.float32))
    plan.c2 = b.add((rng.standard_normal((C2, C1, 7, 7)) * np.sqrt(2.0 / (C1 * 49))).astype(np.float32))
    plan.c3 = b.add((rng.standard_normal((C3, C2, 3, 3)) * np.sqrt(2.0 / (C2 * 9))).astype(np.float32))
    return b.bytes(), plan


def make_audio(seed: int, seconds: float) -> np.ndarray:
    """16 kHz int16: 5 seeded sinusoids (80-4000 Hz, amplitude U(0.05,0.3)) + N(0, 0.02^2)."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * SR))
    tt = np.arange(n, dtype=np.float64) / SR
    x = np.zeros(n, np.float64)
    for _ in range(5):
        f = rng.uniform(80.0, 4000.0)
        a = rng.uniform(0.05, 0.3)
        ph = rng.uniform(0, 2 * np.pi)
        x += a * np.sin(2 * np.pi * f * tt + ph)
    x += rng.normal(0.0, 0.02, size=n)
    peak = max(np.max(np.abs(x)), 1e-9)
    return np.clip(np.round(x / peak * 0.9 * 32767.0), -32768, 32767).astype(np.int16)


def config_lengths(cfg: int, seed: int = 0) -> list[float]:
    """Utterance lengths in seconds: config 2 (one 58.65 s utterance), config 3 (64 in
    U[2,60] s), config 4 (512 in U[1,13] s rescaled to sum to 3600 s)."""
    rng = np.random.default_rng(1000 + seed)
    if cfg == 2:
        return [58.65]
    if cfg == 3:
        return list(rng.uniform(2.0, 60.0, size=64))
    if cfg == 4:
        l = rng.uniform(1.0, 13.0, size=512)
        return list(l * (3600.0 / l.sum()))
    raise ValueError(cfg)


def lpt_shards(lengths, n_shards: int) -> list[list[int]]:
    """Length-balanced assignment (longest processing time first): each utterance, longest
    first, goes to the shard with the least total length so far."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    loads = [0.0] * n_shards
    shards: list[list[int]] = [[] for _ in range(n_shards)]
    for i in order:
        s = min(range(n_shards), key=lambda j: (loads[j], j))
        shards[s].append(i)
        loads[s] += lengths[i]
    for s in shards:
        s.sort()
    return shards
