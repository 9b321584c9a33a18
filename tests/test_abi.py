"""CPU tests of the C-ABI library: it loads, exports every symbol include/*.h declares, and its
host-only entry points (fbank, CTC collapse) match the oracle.  No GPU compute here."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("wtlgpu.h", "wasr.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(w[pk]_\w+|wasr_\w+)\s*\(", src, re.M):
            names.add(m.group(1))
    return names


def test_library_builds_and_loads(pkg):
    from importlib import import_module  # noqa: F401
    build = pkg.build if hasattr(pkg, "build") else None
    import importlib
    b = importlib.import_module("wechat_asr_gpu_b200.build")
    path = b.build()
    assert os.path.exists(path)
    lib = pkg.abi.load()
    assert lib.wp_version().decode().startswith("wasr-b200")
    assert lib.wk_version()
    assert lib.wasr_version()
    del build


def test_exports_every_declared_symbol(pkg):
    lib_path = pkg.abi.LIB_PATH
    assert os.path.exists(lib_path)
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    decl = declared_functions()
    assert len(decl) >= 50
    missing = decl - exported
    assert not missing, missing
    # and every declared symbol has a ctypes signature in abi.py
    assert decl <= set(pkg.abi.SIGNATURES), decl - set(pkg.abi.SIGNATURES)
    lib = ctypes.CDLL(lib_path)
    for name in decl:
        getattr(lib, name)


def test_reference_binding_symbols_present(pkg):
    """The 23 symbols the reference's Rust shell imports (src/gpu.rs:13-86)."""
    need = """wp_create wp_destroy wp_alloc wp_free wp_h2d wp_d2h wp_devptr wp_sync wp_gemm wp_stream
    wp_capture_begin wp_capture_end wp_replay wp_graph_free wp_graph_count wk_attention_fast wk_front
    wk_norm_quant wk_add_norm_quant wk_quant wk_gelu_quant wk_add wk_argmax""".split()
    assert len(need) == 23
    lib = pkg.abi.load()
    for n in need:
        getattr(lib, n)


def test_product_fbank_bit_exact_vs_oracle(pkg, orc):
    for seed, sec in ((1, 0.5), (2, 3.7)):
        pcm = pkg.synth.make_audio(seed, sec)
        f1, s1 = pkg.fbank(pcm)
        f2, s2 = orc.fbank(pcm)
        np.testing.assert_array_equal(f1, f2)
        np.testing.assert_array_equal(s1, s2)
    f, _ = pkg.fbank(np.zeros(100, np.int16))
    assert f.shape[0] == 0


def test_product_ctc_matches_oracle(pkg, orc):
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 4, size=500).astype(np.uint32)
    np.testing.assert_array_equal(pkg.ctc_collapse(ids), orc.ctc(ids))


def test_host_argument_errors_without_gpu(pkg):
    """Argument checks that return before any CUDA call (csrc/wtlgpu.cu:536-538 order)."""
    L = pkg.abi.load()
    assert L.wp_gemm(None, None, None, 1, 1, 0, 1, 1.0, 2 ** 64 - 1, None) == -1
    assert L.wp_quant_rows(None, 1, 1, None, None, None) == -1
    assert L.wp_sync(None) == -1
    assert L.wp_set_stream(None, None) == -1
    assert L.wp_devptr(None, 0) is None
    assert L.wp_graph_count(None) == 0
    assert L.wp_is_capturing(None) == 0
    assert L.wp_capture_begin(None) == -1
    assert L.wp_replay(None, None) == -1
    assert L.wp_graph_free(None, None) == 0
    assert L.wk_attention_fast(None, None, None, None, 4, 512, 8, None, None) == -1
    assert L.wasr_forward(None, None, None, 0, None, None, 0) == -1
    assert L.wasr_model_create(None, 0, None, 0, 16) is None


def test_lpt_shards_balance(pkg):
    lens = pkg.synth.config_lengths(4)
    assert len(lens) == 512 and abs(sum(lens) - 3600.0) < 1e-6
    assert min(lens) >= 0.99 and max(lens) <= 13.1
    for n in (1, 2, 4, 8):
        sh = pkg.synth.lpt_shards(lens, n)
        assert sorted(i for s in sh for i in s) == list(range(512))
        loads = [sum(lens[i] for i in s) for s in sh]
        assert max(loads) - min(loads) <= max(lens)
