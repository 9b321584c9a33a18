"""The reference's model directory (.xnet + dict.decoder.utf8.txt), CPU only.

* A synthetic 40-layer model written by `xnet.write_model_dir` parses with the restated
  src/xnet.rs parser and loads back through the restated build_plan into exactly the blob and
  plan it was made from, so the engine runs the same weights from the reference's file format.
* The written file meets every structural check of the reference's parser (magic, >100
  records, byte length = product of dims x element size, terminator + at most 16 zero bytes),
  and the names, dtypes and shapes that Model::load asks for (src/model.rs:240-305).
* Malformed files are rejected the way the reference rejects them.
"""
import os
import struct

import numpy as np
import pytest


@pytest.fixture(scope="module")
def model_dir(pkg, tmp_path_factory):
    blob, plan = pkg.synth.make_model(seed=5, n_layers=40)
    d = str(tmp_path_factory.mktemp("xnet_model"))
    pkg.xnet.write_model_dir(d, blob, plan)
    return d, blob, plan


def test_roundtrip_blob_and_plan(pkg, model_dir):
    d, blob, plan = model_dir
    blob2, plan2, tokens = pkg.xnet.load_plan(d)
    assert blob2.size == blob.size
    assert np.array_equal(blob2, blob)
    assert bytes(plan2) == bytes(plan)
    assert len(tokens) == plan.vocab and tokens[3] == "t3"


def test_reference_structure_and_names(pkg, model_dir):
    d, blob, plan = model_dir
    raw = open(os.path.join(d, "model.xnet"), "rb").read()
    assert raw[:4] == b"XNET"
    recs = pkg.xnet.parse(raw)
    assert len(recs) > 100
    assert raw[-16:] == struct.pack("<I", 0) + bytes(12)       # terminator + zero padding
    X = pkg.xnet
    for i in (0, 39):
        r = recs[f"layers.{i}.attention.q_conv.weight_quantized_s8"]
        assert r.dtype == X.I8 and r.dims == [512, 512] and r.scale is not None
        assert recs[f"layers.{i}.feed_forward.filter_conv.weight_quantized_s8"].dims == [2048, 512]
        assert recs[f"layers.{i}.feed_forward.output_conv.weight_quantized_s8"].dims == [512, 2048]
        assert recs[f"layers.{i}.prior_norm.weight"].dtype == X.F32
    assert recs["output_conv.weight_quantized_s8"].dims == [plan.vocab, 512]
    assert recs["output_conv.bias"].dims == [plan.vocab]
    assert recs["frontend.linear.weight_quantized_s8"].dims == [512, 3840]
    assert recs["frontend.conv2d_1.weight"].dims == [64, 32, 7, 7]
    for r in recs.values():
        assert r.len == int(np.prod(r.dims)) * X._ELEM[r.dtype]
    # a quantised tensor's bytes are the blob's bytes
    r = recs["layers.7.attention.v_conv.weight_quantized_s8"]
    m = plan.layers[7].v
    assert raw[r.off:r.off + r.len] == blob[m.off:m.off + r.len].tobytes()
    assert np.float32(r.scale) == np.float32(m.s)


def test_malformed_files_rejected(pkg, model_dir, tmp_path):
    d, _, _ = model_dir
    raw = open(os.path.join(d, "model.xnet"), "rb").read()
    X = pkg.xnet
    with pytest.raises(ValueError):
        X.parse(b"XNEX" + raw[4:])                 # wrong magic
    with pytest.raises(ValueError):
        X.parse(raw[:len(raw) // 2])               # truncated: no chain reaches the end
    with pytest.raises(ValueError):
        X.parse(raw + bytes(32))                   # more than 16 bytes after the terminator
    # a dictionary that does not match the output layer
    bad = tmp_path / "m"
    bad.mkdir()
    (bad / "model.xnet").write_bytes(raw)
    (bad / "dict.decoder.utf8.txt").write_text("0 a\n1 b\n")
    with pytest.raises(ValueError):
        X.load_plan(str(bad))


def test_non_reference_plans_refused(pkg):
    blob, plan = pkg.synth.make_model(seed=6, n_layers=2)
    with pytest.raises(ValueError):
        pkg.xnet.tensors_from_blob(blob, plan)     # the reference loader needs 40 layers
