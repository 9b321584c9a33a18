"""Regenerate the committed golden fixtures from the CPU oracle (the restatement of the
reference CPU path; see oracle/wasr_oracle.h).

  kat0.npz      inputs and outputs of the reference's only known-answer test,
                src/kernels.rs:185-208 (LCG seed 7, t=5 k=64 n=11, ws=0.5, bias[j]=j)
  fwd_small.npz a 2-layer random-init model (synth.make_model(seed=3, n_layers=2)) on the fbank
                of 1.3 s of synthetic audio (synth.make_audio(seed=21)): per-frame ids, the
                top-5 logits of every frame and the full logits of frames 0 and 7

Run:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from conftest import load_oracle, load_pkg  # noqa: E402
from test_oracle import kat0_inputs  # noqa: E402


def main():
    orc = load_oracle()
    orc.build()
    pkg = load_pkg()
    t, k, n, x, w, b = kat0_inputs()
    q, s = orc.quant(x)
    out = orc.qgemm(q, s, w, 0.5, bias=b)
    np.savez(os.path.join(HERE, "kat0.npz"), x=x, w=w, q=q, s=s, out=out)

    blob, plan = pkg.synth.make_model(seed=3, n_layers=2)
    pcm = pkg.synth.make_audio(21, 1.3)
    feats, sil = orc.fbank(pcm)
    ids, lo = orc.forward(blob, plan, feats, want_logits=True)
    top = -np.sort(-lo, axis=1)[:, :5]
    np.savez(os.path.join(HERE, "fwd_small.npz"), feats=feats, ids=ids, top5=top, logits0=lo[0], logits7=lo[7])
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
