"""GPU fbank (wasr_fbank_device) against the host fbank (wasr_fbank, the src/fbank.rs
restatement that tests/test_oracle.py pins against the oracle), batched over ragged utterances:
shorter than one window (no frames), exactly one window, frame-boundary lengths, up to 30 s,
digital silence and full-scale clipping.

Bar: the f32 features and silence frames are identical.  CUDA's double log may differ from the
host libm's in the last place; that reaches an f32 value only when the f64 value sits on an f32
rounding boundary, so up to 1e-6 of the values may be one f32 ulp apart (none were in practice:
the test prints the count).
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


def test_gpu_fbank_matches_host(pkg, gpu_lib, dev):
    L = gpu_lib
    pcms = _utterances(pkg)
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
    ref = np.concatenate([h[0] for h in host if h[0].size], 0) if frames else np.zeros((0, 40), np.float32)
    ref_sil = np.stack([h[1] for h in host])
    assert [h[0].shape[0] for h in host] == nfr
    diff = feats.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64)
    off = int(np.count_nonzero(diff))
    print(f"fbank: {frames} frames x 40, values differing: {off}")
    assert np.all(np.abs(diff) <= 1)
    assert off <= max(1, int(1e-6 * feats.size))
    np.testing.assert_array_equal(sil, ref_sil)


def test_gpu_fbank_null_and_empty(pkg, gpu_lib, dev):
    L = gpu_lib
    assert L.wasr_fbank_device(None, None, None, 0, 0, None, None, None, None) == 0   # nothing to do
    p = dev.empty(64)
    assert L.wasr_fbank_device(None, p, p, 1, 0, p, p, p, None) == -1
