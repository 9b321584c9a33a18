"""The streaming front end and text output (src/stream.rs, src/model.rs:620-642), CPU only.

* The library's streaming fbank (wasr_fbank_stream_*) gives, for any split of a signal into
  pushes, the frames of the whole-signal fbank, and after each push the silence frame of the
  prefix's rolling mean (the oracle's whole-prefix fbank).
* text / tidy of the package equal the oracle's C restatements on random id sequences over a
  vocabulary with every kind of token, and the hand-derived cases below.
* The dictionary is split into lines the way Rust's str::lines splits them.
* Stream's schedule (push's commit loop, partial, finish) driven by the oracle's forward gives
  the oracle Stream's ids after every push, at both the whole-utterance and the block path.
"""
import numpy as np
import pytest


class OracleEngine:
    """The oracle's forward behind the engine interface Stream uses."""

    def __init__(self, orc, blob, plan):
        self.orc, self.blob, self.plan = orc, blob, plan
        self.graph_calls = []

    def forward(self, windows):
        return [self.orc.forward(self.blob, self.plan, w) for w in windows]

    def set_graphs(self, on):
        self.graph_calls.append(bool(on))


def test_fbank_stream_any_split_equals_whole(pkg, orc):
    st = pkg.stream
    rng = np.random.default_rng(3)
    pcm = pkg.synth.make_audio(7, 3.0)
    whole, sil_whole = orc.fbank(pcm)
    for trial in range(3):
        fb = st.Fbank()
        cuts = np.sort(rng.integers(0, pcm.size, 12 + 8 * trial))
        pieces = np.split(pcm, cuts)
        pieces.insert(3, pcm[:0])  # an empty push
        got, done = [], 0
        for p in pieces:
            got.append(fb.push(p))
            done += p.size
            ref_f, ref_sil = orc.fbank(pcm[:done])
            assert np.array_equal(np.concatenate(got, 0), ref_f)
            if ref_f.shape[0]:
                assert np.array_equal(fb.silence(), ref_sil)
        assert np.array_equal(np.concatenate(got, 0), whole)
        assert np.array_equal(fb.silence(), sil_whole)
        fb.close()
    # one sample at a time across the first frames
    fb = st.Fbank()
    got = [fb.push(pcm[i:i + 1]) for i in range(1200)]
    assert np.array_equal(np.concatenate(got, 0), orc.fbank(pcm[:1200])[0])


def _vocab():
    toks = ["<blank>", "<UNK>", "<SPACE>", "|", "", "|hello", "|world", "|x", "|中国", "ok", "2", "a",
            "，", "。", "？", "！", "、", ",", ".", "?", "!", "你", "好", "世界", "|A1"]
    return toks


@pytest.mark.parametrize("seed", range(4))
def test_text_and_tidy_vs_oracle(pkg, orc, seed):
    st = pkg.stream
    vocab = _vocab()
    rng = np.random.default_rng(seed)
    for _ in range(200):
        n = int(rng.integers(0, 40))
        ids = rng.integers(0, len(vocab), n).astype(np.uint32)
        rep = rng.random(n) < 0.3  # repeats and blanks, as CTC output has them
        for i in range(1, n):
            if rep[i]:
                ids[i] = ids[i - 1]
        ids[rng.random(n) < 0.2] = 0
        t = st.text(ids, vocab)
        assert t == orc.text(ids, vocab)
        assert st.tidy(t) == orc.tidy(t)
        assert st.tidy(t).rstrip(st.PUNCT) == orc.tidy(t, trim_end=True)


def test_text_known_answers(pkg):
    st = pkg.stream
    v = _vocab()
    ix = {t: i for i, t in enumerate(v)}
    T = lambda *toks: st.text([ix[t] if isinstance(t, str) else t for t in toks], v)  # noqa: E731
    assert T("你", "你", "<blank>", "你", "好") == "你你好"                 # repeats collapse, blank splits
    assert T("<UNK>", "你") == "你"
    assert T("ok", "|hello") == "ok hello"                                  # ASCII letter before a word start
    assert T("2", "|hello") == "2 hello"                                    # ASCII digit too
    assert T("你", "|hello", "|world") == "你hello world"
    assert T("<SPACE>", "|hello") == " hello"
    assert T("|", "|hello") == "|hello"                                     # "|" alone is a plain token
    assert T("|中国", "|hello") == "中国hello"                              # last char not ASCII
    assert T("|A1", "|x") == "A1 x"
    assert T("", "a") == "a"
    assert st.tidy("，。你好，，世界！！") == "你好，世界！"
    assert st.tidy("!?,") == ""
    assert st.tidy("a.,b") == "a,b"
    assert st.tidy("你好。").rstrip(st.PUNCT) == "你好"


def test_vocab_lines_like_rust(pkg, tmp_path):
    p = tmp_path / "dict.decoder.utf8.txt"
    p.write_bytes(b"0 <blank>\r\n1 \xe4\xbd\xa0\n2 a b\n3\n4 x y\r\r\n5 \n")
    # lines(): "0 <blank>", "1 ni", "2 a b", "3", "4 x y\r" (one CR removed), "5 "
    assert pkg.stream.load_vocab(str(p)) == ["<blank>", "\u4f60", "a", "", "x", ""]
    # U+2028 and VT are not line ends for str::lines
    p.write_bytes(b"0 a\xe2\x80\xa8b\n1 c\x0bd\n")
    assert pkg.stream.load_vocab(str(p)) == ["a\u2028b", "c\x0bd"]
    p.write_bytes(b"0 a\n1 b")
    assert pkg.stream.load_vocab(str(p)) == ["a", "b"]
    p.write_bytes(b"")
    assert pkg.stream.load_vocab(str(p)) == []
    p.write_bytes(b"0 \xff\n")
    with pytest.raises(UnicodeDecodeError):
        pkg.stream.load_vocab(str(p))


def test_env_frames(pkg, monkeypatch):
    st = pkg.stream
    for v, want in [("400", 400), ("+300", 300), ("99", 200), (" 400", 200), ("4e2", 200), ("", 200),
                    ("1000", 1000)]:
        monkeypatch.setenv("WTL_PREV", v)
        assert st._env_frames("WTL_PREV", 200) == want, v


@pytest.fixture(scope="module")
def small_model(pkg):
    return pkg.synth.make_model(seed=21, n_layers=2)


@pytest.mark.parametrize("seconds,chunk", [(12.0, 1600), (26.0, 4000)])
def test_stream_schedule_vs_oracle(pkg, orc, small_model, seconds, chunk):
    """Package Stream (streaming fbank + schedule) and oracle Stream (whole-prefix fbank + C
    schedule) over the oracle's forward: identical partial ids after every push and identical
    finish ids (12 s: the whole-utterance finish; 26 s: committed blocks + tail)."""
    blob, plan = small_model
    pcm = pkg.synth.make_audio(31, seconds)
    eng = OracleEngine(orc, blob, plan)
    s = pkg.stream.Stream(eng, prev=200, blk=400, post=100)
    o = orc.Stream(blob, plan, prev=200, blk=400, post=100)
    assert eng.graph_calls == [False]
    for k, a in enumerate(range(0, pcm.size, chunk)):
        s.push(pcm[a:a + chunk])
        o.push(pcm[a:a + chunk])
        assert s.s == o.s.value and list(s.ids) == o.ids[:o.n_ids.value].tolist()
        if k % 3 == 2:
            assert np.array_equal(s.partial_ids(), o.partial())
            assert s.fresh() == 0
    assert np.array_equal(s.finish_ids(), o.finish())
    if seconds > 20:
        assert s.s > 0  # blocks were committed


def test_stream_text_vs_oracle(pkg, orc, small_model):
    blob, plan = small_model
    rng = np.random.default_rng(5)
    base = _vocab()  # every output id spells as one of the token kinds
    vocab = [base[0]] + [base[int(rng.integers(1, len(base)))] for _ in range(plan.vocab - 1)]
    pcm = pkg.synth.make_audio(33, 22.0)
    eng = OracleEngine(orc, blob, plan)
    s = pkg.stream.Stream(eng, vocab, prev=200, blk=400, post=100)
    o = orc.Stream(blob, plan, vocab, prev=200, blk=400, post=100)
    for a in range(0, pcm.size, 16000):
        s.push(pcm[a:a + 16000])
        o.push(pcm[a:a + 16000])
        assert s.partial() == o.partial()
    assert s.finish() == o.finish()
