"""The streaming front end on the B200 engine (src/stream.rs:58-168): the package Stream over
host.Engine (40-layer synthetic model, the GPU forward per window) against the oracle Stream
(whole-prefix fbank, C schedule, CPU forward): the same ids after every push, the same
partial ids and finish ids, and the same text through Model::text / tidy."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model40(pkg):
    return pkg.synth.make_model(seed=41, n_layers=40)


@pytest.fixture(scope="module")
def engine(pkg, gpu_lib, model40):
    blob, plan = model40
    e = pkg.Engine(blob, plan, max_rows=4096)
    yield e
    e.close()


def test_stream_partials_vs_oracle(pkg, orc, model40, engine):
    blob, plan = model40
    pcm = pkg.synth.make_audio(51, 24.0)
    s = pkg.stream.Stream(engine, prev=200, blk=400, post=100)
    o = orc.Stream(blob, plan, prev=200, blk=400, post=100)
    chunk = 8000  # 0.5 s
    for k, a in enumerate(range(0, pcm.size, chunk)):
        s.push(pcm[a:a + chunk])
        o.push(pcm[a:a + chunk])
        assert s.s == o.s.value and list(s.ids) == o.ids[:o.n_ids.value].tolist()
        if k % 4 == 3:
            assert np.array_equal(s.partial_ids(), o.partial())
    assert s.s > 0
    assert np.array_equal(s.finish_ids(), o.finish())
    assert s.n_windows == o.n_fwd


def test_transcribe_text_vs_oracle(pkg, orc, model40, engine):
    blob, plan = model40
    rng = np.random.default_rng(9)
    vocab = ["<blank>"] + [["你", "好", "，", "。", "|hi", "<SPACE>", "<UNK>", "a"][int(rng.integers(0, 8))]
                           for _ in range(plan.vocab - 1)]
    for seconds in (6.0, 23.0):  # the whole-utterance finish, and blocks + tail
        pcm = pkg.synth.make_audio(61 + int(seconds), seconds)
        got = pkg.stream.transcribe(engine, pcm, vocab)
        o = orc.Stream(blob, plan, vocab, prev=200, blk=400, post=100)
        o.push(pcm)
        assert got == o.finish()
