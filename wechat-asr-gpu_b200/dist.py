"""Utterance-sharded batch transcription across the GPUs of one node (one process per GPU).

Utterances are independent (the reference decodes them one after another, src/bin/wasr.rs:147-169),
so the node-level driver only has to split them and collect the results:

* every rank takes a length-balanced LPT shard (``synth.lpt_shards``) and transcribes it on its
  own device and stream;
* results go through the rendezvous key-value store, not through a collective: each rank writes
  ``wasr/res/<rank>``, and the gathering rank waits for each key with a deadline;
* a rank that never delivers (raised, exited or hung) is detected on the host when its key times
  out, and its utterances are re-queued to the gathering rank, which transcribes them itself.
  No GPU kernel waits on another rank, so a dead rank can never leave a kernel spinning.

``run_sharded`` is used by the tests with ``gloo`` ranks on CPU (the transcribe function is a
parameter); on a GPU node each rank passes its engine's ``transcribe``.
"""
from __future__ import annotations

import datetime
import io
import pickle
from typing import Callable, Sequence

import numpy as np

from .synth import lpt_shards


def _pack(ids: dict[int, np.ndarray]) -> bytes:
    buf = io.BytesIO()
    pickle.dump({int(k): np.asarray(v, np.uint32) for k, v in ids.items()}, buf, protocol=4)
    return buf.getvalue()


def _unpack(b: bytes) -> dict[int, np.ndarray]:
    return pickle.loads(b)


def run_sharded(transcribe: Callable[[Sequence[int]], list[np.ndarray]], lengths: Sequence[float],
                rank: int, world: int, store, timeout_s: float = 30.0, gather_rank: int = 0,
                tag: str = "wasr") -> list[np.ndarray] | None:
    """Transcribe this rank's LPT shard with ``transcribe(indices) -> ids per index`` and collect
    every utterance's ids on ``gather_rank`` (returned there, in input order; None elsewhere).

    ``store`` is a torch.distributed Store (the process group's rendezvous store).  A rank whose
    result does not appear within ``timeout_s`` is treated as failed and its shard is
    transcribed by the gathering rank."""
    shards = lpt_shards(list(lengths), world)
    mine = shards[rank]
    local = dict(zip(mine, transcribe(mine))) if mine else {}
    if rank != gather_rank:
        store.set(f"{tag}/res/{rank}", _pack(local))
        return None
    out: dict[int, np.ndarray] = dict(local)
    failed: list[int] = []
    for r in range(world):
        if r == gather_rank:
            continue
        key = f"{tag}/res/{r}"
        try:
            store.wait([key], datetime.timedelta(seconds=timeout_s))
            out.update(_unpack(store.get(key)))
        except Exception:  # the rank died, hung or never joined: re-queue its utterances
            failed.append(r)
    for r in failed:
        redo = shards[r]
        if redo:
            out.update(dict(zip(redo, transcribe(redo))))
    missing = [i for i in range(len(lengths)) if i not in out]
    if missing:
        raise RuntimeError(f"utterances without a result: {missing[:8]}")
    run_sharded.last_failed = failed
    return [out[i] for i in range(len(lengths))]


run_sharded.last_failed = []
