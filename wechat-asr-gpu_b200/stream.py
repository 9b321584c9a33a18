"""The reference's streaming front end (src/stream.rs) and text output (src/model.rs:620-642)
over the GPU engine.

* `text(ids, vocab)` -- Model::text: CTC collapse (repeats and blank 0 dropped), then the
  vocabulary's spelling: "<UNK>" is dropped, "<SPACE>" is a space, a token "|w" starts an
  English word (with a space first when the text so far ends in an ASCII letter or digit).
* `tidy(s)` -- src/stream.rs:203-210: leading punctuation removed; of two adjacent
  punctuation marks only the second kept.
* `load_vocab(path)` -- the dictionary as Model::load reads it (src/model.rs:267-271): lines
  split like Rust's `str::lines`, the token is the second space-separated field.
* `Fbank` -- the streaming fbank (src/fbank.rs:122-161) of the library (wasr_fbank_stream_*).
* `Stream` -- Stream::push / partial / finish (src/stream.rs:58-168): blocks of `blk` frames
  are committed once `post` frames of right context exist, each decoded with `prev` frames of
  left context and 50 silence frames; partial() re-decodes the open tail with half the left
  context and trims trailing punctuation; finish() decodes an utterance of at most 2000 frames
  in one piece.  Windows go through `engine.forward` one at a time, as in the reference.
* `transcribe(engine, pcm, vocab)` -- the library entry of src/lib.rs:57-67 (push + finish).
"""
from __future__ import annotations

import os
import re

import numpy as np

from . import abi, xnet

PREV_DEFAULT, BLK_DEFAULT, POST_DEFAULT = 200, 400, 100   # src/stream.rs:11-13
PAD = 50                                                  # src/stream.rs:15
WHOLE_MAX = 2000                                          # src/stream.rs:17
GRAPH_MIN_FRAMES = 20000                                  # src/stream.rs:19
PUNCT = "，。？！、,.?!"                                   # src/stream.rs:173
_ALNUM = set("0123456789abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ")


def text(ids, vocab) -> str:
    """Model::text (src/model.rs:620-642)."""
    out: list[str] = []
    last = ""  # last character appended
    prev = None
    for i in (int(v) for v in ids):
        if i != prev and i != 0:
            t = vocab[i]
            if t == "<UNK>":
                pass
            elif t == "<SPACE>":
                out.append(" ")
                last = " "
            elif len(t) > 1 and t.startswith("|"):
                if last in _ALNUM:
                    out.append(" ")
                out.append(t[1:])
                last = t[-1] if len(t) > 1 else last
            else:
                out.append(t)
                last = t[-1] if t else last
        prev = i
    return "".join(out)


def tidy(s: str) -> str:
    """src/stream.rs:203-210."""
    c = s.lstrip(PUNCT)
    return "".join(ch for i, ch in enumerate(c) if not (ch in PUNCT and i + 1 < len(c) and c[i + 1] in PUNCT))


def load_vocab(path: str) -> list[str]:
    """dict.decoder.utf8.txt as Model::load reads it (src/model.rs:267-271)."""
    return xnet.read_vocab(path)


_USIZE = re.compile(r"^\+?[0-9]+$")


def _env_frames(key: str, default: int) -> int:
    """src/stream.rs:30-33: a usize from the environment, used only when >= 100."""
    v = os.environ.get(key)
    if v is None or not _USIZE.match(v):
        return default
    n = int(v)
    return n if 100 <= n < (1 << 64) else default


class Fbank:
    """The streaming fbank (src/fbank.rs:122-161 Fbank) of the library."""

    def __init__(self):
        self.L = abi.load()
        self.st = self.L.wasr_fbank_stream_create()
        if not self.st:
            raise MemoryError("wasr_fbank_stream_create")

    def close(self):
        if self.st:
            self.L.wasr_fbank_stream_destroy(self.st)
            self.st = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def push(self, pcm) -> np.ndarray:
        """Append samples; returns the frames they complete, [k][40] fp32."""
        pcm = np.ascontiguousarray(pcm, np.int16)
        k = int(self.L.wasr_fbank_stream_pending(self.st, pcm.size))
        out = np.zeros((max(k, 1), abi.DIM), np.float32)
        got = int(self.L.wasr_fbank_stream_push(self.st, pcm.ctypes.data, pcm.size, out.ctypes.data, k))
        if got != k:
            raise RuntimeError(f"wasr_fbank_stream_push rc={got}")
        return out[:k]

    def silence(self) -> np.ndarray:
        sil = np.zeros(abi.DIM, np.float32)
        if self.L.wasr_fbank_stream_silence(self.st, sil.ctypes.data):
            raise RuntimeError("wasr_fbank_stream_silence")
        return sil


class Stream:
    """Stream (src/stream.rs:37-168) over an engine: any object with `forward(windows)` giving
    one id array per window (host.Engine; the oracle in the CPU tests) and, optionally,
    `set_graphs(on)`.  vocab None: partial() / finish() return ids, else text."""

    def __init__(self, engine, vocab=None, prev: int | None = None, blk: int | None = None,
                 post: int | None = None):
        self.engine, self.vocab = engine, vocab
        self.prev = prev if prev is not None else _env_frames("WTL_PREV", PREV_DEFAULT)
        self.blk = blk if blk is not None else _env_frames("WTL_BLK", BLK_DEFAULT)
        self.post = post if post is not None else _env_frames("WTL_POST", POST_DEFAULT)
        self.fb = Fbank()
        self._feats = np.zeros((1024, abi.DIM), np.float32)
        self.n = 0          # frames so far
        self.ids: list[int] = []
        self.s = 0          # commit position (frames)
        self._fresh = 0
        self.n_windows = 0  # forwards run (commit, partial, finish)
        self._graphs(False)  # Stream::new (src/stream.rs:47-50)

    def _graphs(self, on: bool):
        f = getattr(self.engine, "set_graphs", None)
        if f is not None:
            f(on)

    @property
    def feats(self) -> np.ndarray:
        return self._feats[:self.n]

    def fresh(self) -> int:
        """Frames added since the last partial()."""
        return self._fresh

    def push(self, pcm):
        """src/stream.rs:58-70."""
        new = self.fb.push(pcm)
        k = new.shape[0]
        if self.n + k > self._feats.shape[0]:
            grown = np.zeros((max(2 * self._feats.shape[0], self.n + k), abi.DIM), np.float32)
            grown[:self.n] = self._feats[:self.n]
            self._feats = grown
        self._feats[self.n:self.n + k] = new
        self.n += k
        if self.n >= GRAPH_MIN_FRAMES:
            self._graphs(True)
        self._fresh += k
        while self.n >= self.s + self.blk + self.post:
            self._commit()

    def _decode(self, prev: int, end: int, pad: int) -> np.ndarray:
        """src/stream.rs:128-134: [s - prev, end) plus pad silence frames; ids from s on."""
        a = max(self.s - prev, 0)
        sil = self.fb.silence()
        x = np.concatenate([self._feats[a:end], np.broadcast_to(sil, (pad, abi.DIM))], 0)
        out = self.engine.forward([np.ascontiguousarray(x, np.float32)])[0]
        self.n_windows += 1
        return np.asarray(out[(self.s - a) // 5:], np.uint32)

    def _commit(self):
        """src/stream.rs:136-147."""
        ids = self._decode(self.prev, self.s + self.blk + self.post, PAD)[: self.blk // 5]
        m = len(ids)
        for c in range(m - 1, m // 2 - 1, -1):  # the last blank pair in the second half
            if c >= 1 and ids[c] == 0 and ids[c - 1] == 0:
                m = c
                break
        ids = ids[:m]
        self.s += len(ids) * 5
        self.ids.extend(int(v) for v in ids)

    def partial_ids(self) -> np.ndarray:
        """The ids behind partial(): committed + the open tail with half the left context."""
        self._fresh = 0
        ids = list(self.ids)
        if self.n > self.s:
            ids.extend(int(v) for v in self._decode(self.prev // 2, self.n, PAD))
        return np.array(ids, np.uint32)

    def partial(self):
        """src/stream.rs:150-157."""
        ids = self.partial_ids()
        return ids if self.vocab is None else tidy(text(ids, self.vocab)).rstrip(PUNCT)

    def finish_ids(self) -> np.ndarray:
        """The ids behind finish() (src/stream.rs:159-168)."""
        if self.n <= WHOLE_MAX:
            self.n_windows += 1
            if self.n < 5:
                return np.zeros(0, np.uint32)
            return np.asarray(self.engine.forward([np.ascontiguousarray(self.feats, np.float32)])[0], np.uint32)
        ids = list(self.ids)
        if self.n > self.s:
            ids.extend(int(v) for v in self._decode(self.prev, self.n, PAD))
        return np.array(ids, np.uint32)

    def finish(self):
        ids = self.finish_ids()
        return ids if self.vocab is None else tidy(text(ids, self.vocab))


def transcribe(engine, pcm, vocab=None):
    """src/lib.rs:57-67 (CUDA / CPU backends): push the whole utterance, then finish."""
    s = Stream(engine, vocab)
    s.push(pcm)
    out = s.finish()
    s.fb.close()
    return out
