"""Multi-rank host logic on CPU: two ``gloo`` ranks run the utterance-sharded driver
(``dist.run_sharded``) with the oracle standing in for each rank's GPU engine.

* normal run: the gathered per-utterance ids equal a single-process transcription;
* failure: rank 1 raises before delivering its shard; rank 0 detects it on the host when the
  result key times out, re-queues rank 1's utterances and still returns every utterance.
"""
import datetime
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _workload():
    sys.path.insert(0, HERE)
    from conftest import load_oracle, load_pkg
    pkg, orc = load_pkg(), load_oracle()
    orc.set_threads(1)
    blob, plan = pkg.synth.make_model(seed=9, n_layers=1)
    lengths = [0.6, 1.4, 0.3, 1.1, 0.8, 0.5, 1.2]
    data = []
    for i, L in enumerate(lengths):
        f, s = orc.fbank(pkg.synth.make_audio(500 + i, L))
        data.append((f, s))

    def transcribe(idx):
        return [orc.transcribe(blob, plan, data[i][0], data[i][1])[0] for i in idx]
    return pkg, lengths, transcribe


def _rank_main(rank, world, port, fail_rank, q):
    import torch.distributed as dist
    pkg, lengths, transcribe = _workload()
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    if rank == fail_rank:
        raise RuntimeError("simulated worker failure before delivering its shard")
    from wechat_asr_gpu_b200.dist import run_sharded
    out = run_sharded(transcribe, lengths, rank, world, store, timeout_s=4.0)
    if rank == 0:
        q.put(([o.tolist() for o in out], list(run_sharded.last_failed)))


def _run(world, fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    try:
        out, failed = q.get(timeout=120)
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out, failed, [p.exitcode for p in ps]


@pytest.fixture(scope="module")
def reference():
    pkg, lengths, transcribe = _workload()
    return [o.tolist() for o in transcribe(range(len(lengths)))]


def test_two_gloo_ranks_gather_in_order(reference):
    out, failed, codes = _run(2, fail_rank=-1)
    assert failed == []
    assert out == reference
    assert codes == [0, 0]


def test_failed_rank_is_requeued(reference):
    out, failed, codes = _run(2, fail_rank=1)
    assert failed == [1]
    assert out == reference
    assert codes[0] == 0 and codes[1] != 0
