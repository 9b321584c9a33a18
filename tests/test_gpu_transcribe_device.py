"""On-device windowing: wasr_transcribe_device runs the reference window schedule
(src/stream.rs:58-168) on features that stay on the GPU (wasr_fbank_device's output), gathering
each round's windows and silence pads on the device.

Bar: the per-frame ids equal the oracle's transcription (oracle/, the C restatement of the
reference's CPU path and schedule) of the same features, utterance by utterance; and ids and
offsets equal wasr_transcribe's on the same features copied to the host, for a batch that mixes whole-utterance windows with block windows (26 s and 41 s
utterances are longer than the 2000-frame whole-window limit, so their commit and finish
windows carry the 50-frame silence pad), for a batch of whole utterances only (read straight
from the caller's array), at two block sizes, and on a repeated call.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LENS = [0.3, 2.0, 7.3, 26.0, 41.0, 0.01]  # seconds; the first three are whole windows, 0.01 s has no frames


def _frames(n):
    return (n - 400) // 160 + 1 if n >= 400 else 0


@pytest.fixture(scope="module")
def small_model(pkg):
    return pkg.synth.make_model(seed=51, n_layers=2)


def test_transcribe_device_equals_host(pkg, orc, gpu_lib, dev, small_model):
    L = gpu_lib
    pcms = [pkg.synth.make_audio(900 + i, s) for i, s in enumerate(LENS)]
    n = len(pcms)
    soff = np.concatenate([[0], np.cumsum([p.size for p in pcms])]).astype(np.int64)
    nfr = np.array([_frames(p.size) for p in pcms], np.int64)
    foff = np.concatenate([[0], np.cumsum(nfr)]).astype(np.int64)
    frames = int(foff[-1])
    p_pcm, p_soff, p_foff = dev.put(np.concatenate(pcms).astype(np.int16)), dev.put(soff), dev.put(foff)
    p_raw, p_feats, p_sil = dev.empty(frames * 40 * 8), dev.empty(frames * 40 * 4), dev.empty(n * 40 * 4)
    assert L.wasr_fbank_device(p_pcm, p_soff, p_foff, n, frames, p_raw, p_feats, p_sil, None) == 0
    feats = dev.get(p_feats, (frames, 40), np.float32)  # synchronous: the fbank has finished
    sil = dev.get(p_sil, (n, 40), np.float32)
    assert nfr[3] > 2000 and nfr[4] > 2000 and nfr[2] <= 2000 and nfr[5] == 0

    blob, plan = small_model
    eng = pkg.Engine(blob, plan, max_rows=4096)
    try:
        for k, (prev, blk, post) in [(n, (200, 400, 100)), (n, (200, 1600, 100)), (3, (200, 400, 100))]:
            cap = int(nfr[:k].sum() // 5 + 64 * k + 64)
            ids_h, off_h = np.zeros(cap, np.uint32), np.zeros(k + 1, np.int64)
            assert L.wasr_transcribe(eng.m, feats.ctypes.data, nfr.ctypes.data, sil.ctypes.data, k, prev, blk, post,
                                     ids_h.ctypes.data, off_h.ctypes.data, cap) == 0
            assert off_h[-1] > 0
            for _ in range(2):
                ids_d, off_d = np.zeros(cap, np.uint32), np.zeros(k + 1, np.int64)
                assert L.wasr_transcribe_device(eng.m, p_feats, nfr.ctypes.data, p_sil, k, prev, blk, post,
                                                ids_d.ctypes.data, off_d.ctypes.data, cap) == 0
                np.testing.assert_array_equal(off_d, off_h)
                np.testing.assert_array_equal(ids_d[:off_h[-1]], ids_h[:off_h[-1]])
        # the Engine wrappers: per-utterance ids, device features against host features, and
        # both against the oracle's transcription of each utterance
        per_utt = [feats[foff[i]:foff[i + 1]] for i in range(n)]
        want = eng.transcribe(per_utt, list(sil), prev=200, blk=400, post=100)
        got = eng.transcribe_device(p_feats, nfr, p_sil, prev=200, blk=400, post=100)
        assert len(got) == n and all(np.array_equal(a, b) for a, b in zip(got, want))
        for i in range(n):
            ref, _ = orc.transcribe(blob, plan, per_utt[i], sil[i], prev=200, blk=400, post=100)
            np.testing.assert_array_equal(got[i], ref, err_msg=f"utterance {i}")
        for blk in (1600,):
            got = eng.transcribe_device(p_feats, nfr, p_sil, prev=200, blk=blk, post=100)
            for i in range(n):
                ref, _ = orc.transcribe(blob, plan, per_utt[i], sil[i], prev=200, blk=blk, post=100)
                np.testing.assert_array_equal(got[i], ref, err_msg=f"utterance {i}, blk {blk}")
        # return codes shared with wasr_transcribe
        one = np.zeros(1, np.uint32)
        off = np.zeros(n + 1, np.int64)
        assert L.wasr_transcribe_device(eng.m, p_feats, nfr.ctypes.data, p_sil, n, 200, 400, 100, one.ctypes.data,
                                        off.ctypes.data, 1) == -20
        assert L.wasr_transcribe_device(eng.m, None, nfr.ctypes.data, p_sil, n, 200, 400, 100, one.ctypes.data,
                                        off.ctypes.data, 1) == -1
        assert eng.error() == 0
    finally:
        eng.close()
