"""GPU fbank (wasr_fbank_device) against the oracle's fbank (the C restatement of
src/fbank.rs:21-161 in oracle/, test infrastructure) and against the library's host fbank,
batched over ragged utterances: shorter than one window (no frames), exactly one window,
frame-boundary lengths, up to 30 s, digital silence and full-scale clipping.

Bar: the f32 features and silence frames are identical to both, bit for bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _utterances(pkg):
    lens = [0.005, 0.025, 0.0251, 0.3, 1.0, 2.47, 7.3, 30.0]  # seconds
    pcms = [pkg.synth.make_audio(700 + i, L) for i, L in enumerate(lens)]
    pcms.append(np.zeros(16000, np.int16))                        # digital silence
    clip = np.full(8000, 32767, np.int16)
    clip[1::2] = -32768
    pcms.append(clip)                                             # full-scale square wave
    pcms.append(pkg.synth.make_audio(799, 400 / 16000))           # exactly one window
    pcms.append(pkg.synth.make_audio(798, (400 + 160 * 7) / 16000))
    return pcms


def _frames(n):
    return (n - 400) // 160 + 1 if n >= 400 else 0


def test_gpu_fbank_matches_oracle_and_host(pkg, orc, gpu_lib, dev):
    L = gpu_lib
    pcms = _utterances(pkg)
    oracle = [orc.fbank(p) for p in pcms]
    host = [pkg.fbank(p) for p in pcms]
    soff = np.concatenate([[0], np.cumsum([p.size for p in pcms])]).astype(np.int64)
    nfr = [_frames(p.size) for p in pcms]
    foff = np.concatenate([[0], np.cumsum(nfr)]).astype(np.int64)
    frames, n = int(foff[-1]), len(pcms)
    cat = np.concatenate(pcms).astype(np.int16)
    p_pcm, p_soff, p_foff = dev.put(cat), dev.put(soff), dev.put(foff)
    p_raw = dev.empty(max(frames, 1) * 40 * 8)
    p_feats = dev.empty(max(frames, 1) * 40 * 4)
    p_sil = dev.empty(n * 40 * 4)
    # legacy default stream: the synchronous copies below order after it
    assert L.wasr_fbank_device(p_pcm, p_soff, p_foff, n, frames, p_raw, p_feats, p_sil, None) == 0
    feats = dev.get(p_feats, (frames, 40), np.float32)
    sil = dev.get(p_sil, (n, 40), np.float32)
    assert [o[0].shape[0] for o in oracle] == nfr
    for name, ref_list in (("oracle", oracle), ("host", host)):
        ref = np.concatenate([r[0] for r in ref_list if r[0].size], 0) if frames else np.zeros((0, 40), np.float32)
        np.testing.assert_array_equal(feats, ref, err_msg=name)
        np.testing.assert_array_equal(sil, np.stack([r[1] for r in ref_list]), err_msg=name)


def test_gpu_fbank_null_and_empty(pkg, gpu_lib, dev):
    L = gpu_lib
    assert L.wasr_fbank_device(None, None, None, 0, 0, None, None, None, None) == 0   # nothing to do
    p = dev.empty(64)
    assert L.wasr_fbank_device(None, p, p, 1, 0, p, p, p, None) == -1
