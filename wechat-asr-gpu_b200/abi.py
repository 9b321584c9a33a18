"""ctypes bindings of libwasr_gpu.so (the reference-facing wp_*/wk_* ABI plus the additive
wasr_* engine ABI), and the WasrPlan struct shared with the weight-blob packer.

The library is built in-tree by ``build.py``; there is no CPU or Python fallback: loading
fails loudly if the shared object is missing.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwasr_gpu.so")

WASR_NONE = (1 << 64) - 1
D, HEADS, HD, FF, DIM, FLAT = 512, 8, 64, 2048, 40, 3840
C1, C2, C3, W2 = 32, 64, 192, 41
MAX_LAYERS = 40
PREV, POST, PAD, WHOLE_MAX = 200, 100, 50, 2000


class WasrMat(C.Structure):
    """One int8 weight matrix inside the blob (PlanQ, src/model.rs:58-63) + optional
    per-output-channel scale vector."""
    _fields_ = [("off", C.c_uint64), ("scale_off", C.c_uint64), ("s", C.c_float),
                ("n", C.c_int32), ("k", C.c_int32), ("reserved", C.c_int32)]


class WasrLayer(C.Structure):
    """PlanLayer (src/model.rs:65-79) + optional q/k/v/o biases."""
    _fields_ = [("pn_g", C.c_uint64), ("pn_b", C.c_uint64), ("mn_g", C.c_uint64), ("mn_b", C.c_uint64),
                ("q", WasrMat), ("k", WasrMat), ("v", WasrMat), ("o", WasrMat), ("f1", WasrMat),
                ("f2", WasrMat),
                ("qb", C.c_uint64), ("kb", C.c_uint64), ("vb", C.c_uint64), ("ob", C.c_uint64),
                ("f1b", C.c_uint64), ("f2b", C.c_uint64)]


class WasrPlan(C.Structure):
    """Plan (src/model.rs:81-94)."""
    _fields_ = [("n_layers", C.c_int32), ("vocab", C.c_int32), ("out_n", C.c_int32),
                ("reserved", C.c_int32), ("lin", WasrMat), ("out", WasrMat),
                ("lin_b", C.c_uint64), ("out_b", C.c_uint64), ("c1", C.c_uint64),
                ("c2", C.c_uint64), ("c3", C.c_uint64), ("layers", WasrLayer * MAX_LAYERS)]


# every symbol include/wtlgpu.h and include/wasr.h declare: name -> (restype, argtypes)
P, I, F, Z, U64, I64 = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_uint64, C.c_int64
SIGNATURES = {
    # include/wtlgpu.h
    "wp_create": (P, [P, Z]),
    "wp_destroy": (None, [P]),
    "wp_alloc": (P, [Z]),
    "wp_free": (None, [P]),
    "wp_h2d": (I, [P, P, Z]),
    "wp_d2h": (I, [P, P, Z]),
    "wp_devptr": (P, [P, Z]),
    "wp_sync": (I, [P]),
    "wp_set_stream": (I, [P, P]),
    "wp_stream": (P, [P]),
    "wp_scratch_bytes": (Z, [P]),
    "wp_version": (C.c_char_p, []),
    "wp_gemm": (I, [P, P, P, I, I, Z, I, F, Z, P]),
    "wp_gemm2": (I, [P, P, P, I, I, Z, I, F, P, P, P]),
    "wp_gemm_q": (I, [P, P, P, I, I, Z, I, F, P, P, P, P]),
    "wp_gemm_qg": (I, [P, P, P, I, I, Z, I, F, P, P, P, P]),
    "wp_quant_rows": (I, [P, I, I, P, P, P]),
    "wp_capture_begin": (I, [P]),
    "wp_capture_end": (I, [P, C.POINTER(C.c_void_p)]),
    "wp_replay": (I, [P, P]),
    "wp_graph_free": (I, [P, P]),
    "wp_graph_count": (Z, [P]),
    "wp_is_capturing": (I, [P]),
    "wk_front": (None, [P, P, P, P, P, I, I, P, P, P]),
    "wk_norm_quant": (None, [P, P, P, P, I, I, P, P]),
    "wk_add_norm_quant": (None, [P, P, P, P, P, I, I, P, P]),
    "wk_quant": (None, [P, P, I, I, P, P]),
    "wk_gelu_quant": (None, [P, P, I, I, P, P]),
    "wk_add": (None, [P, P, P, I, I]),
    "wk_argmax": (None, [P, P, I, I, P]),
    "wk_version": (C.c_char_p, []),
    "wk_last_error": (I, []),
    "wk_attention_fast": (I, [P, P, P, P, I, I, I, P, P]),
    "wk_attention": (None, [P, P, P, P, I, I, I, P, P]),
    "wk_attention_tiled": (I, [P, P, P, P, I, I, I, P, P]),
    "wk_attention_tiled_tuned": (I, [P, P, P, P, I, I, I, P, I, I]),
    "wk_attention_tiled_version": (C.c_char_p, []),
    "wk_attention_cublas": (I, [P, P, P, P, I, I, I, P, P]),
    "wk_attention_cublas_part": (I, [I, P, P, P, P, I, I, I, P, P]),
    "wk_attention_version": (C.c_char_p, []),
    "wp_gemm2_pc": (I, [P, P, P, I, I, Z, I, P, P, P, P]),
    "wp_gemm_i32": (I, [P, P, I, I, Z, I, P, P]),
    "wp_gemm_i32_wait_probe": (I, [P, P, I, I, Z, I, P, P, C.c_uint64]),
    "wp_gemm_q_noalloc": (I, [P, P, P, I, I, Z, I, F, P, P, P, P]),
    # include/wasr.h
    "wasr_model_create": (P, [P, Z, C.POINTER(WasrPlan), I, I]),
    "wasr_model_destroy": (None, [P]),
    "wasr_model_set_stream": (I, [P, P]),
    "wasr_model_stream": (P, [P]),
    "wasr_model_set_graphs": (I, [P, I]),
    "wasr_model_error": (I, [P]),
    "wasr_model_set_profile": (I, [P, I]),
    "wasr_model_profile": (I, [P, P, P, I]),
    "wasr_model_kernel_launches": (I64, [P]),
    "wasr_forward": (I, [P, P, P, I, P, P, I]),
    "wasr_transcribe": (I, [P, P, P, P, I, I, I, I, P, P, I64]),
    "wasr_transcribe_device": (I, [P, P, P, P, I, I, I, I, P, P, I64]),
    "wasr_fbank": (I64, [P, I64, P, I64, P]),
    "wasr_fbank_device": (I, [P, P, P, I, I64, P, P, P, P]),
    "wasr_fbank_stream_create": (P, []),
    "wasr_fbank_stream_destroy": (None, [P]),
    "wasr_fbank_stream_pending": (I64, [P, I64]),
    "wasr_fbank_stream_push": (I64, [P, P, I64, P, I64]),
    "wasr_fbank_stream_silence": (I, [P, P]),
    "wasr_ctc_collapse": (I64, [P, I64, P]),
    "wasr_eval_math": (I, [I, P, P, I, P]),
    "wasr_gelu_quant": (I, [P, I, I, P, P, I, P]),
    "wasr_conv3_quant": (I, [P, P, P, P, I, I, P, P, P]),
    "wasr_conv1": (I, [P, P, P, I, I, I, P, P]),
    "wasr_conv2": (I, [P, P, P, P, P, I, I, I, P, P]),
    "wasr_gemm_gelu_quant": (I, [P, P, P, F, P, P, I, I, I, P, P, P, P]),
    "wasr_gemm_gelu_quant_wait_probe": (I, [P, P, P, F, P, P, I, I, I, P, P, P, U64, P]),
    "wasr_gelu_cert_scan": (I, [U64, U64, P, P]),
    "wasr_i8_mma_peak": (I, [I, I, P, P]),
    "wasr_version": (C.c_char_p, []),
}

WASR_F_DEVICE = 1
WASR_F_NOSYNC = 2
# kernel classes of wasr_model_profile (include/wasr.h)
KERNEL_CLASSES = ["conv1", "conv2", "conv3", "quant", "gemm_lin", "layernorm", "gemm_qkv", "attention",
                  "gemm_o", "gemm_f1", "gemm_f2", "gemm_out_argmax", "ids", "gelu_quant"]

_lib = None


def load(path: str | None = None) -> C.CDLL:
    """Load libwasr_gpu.so (once) and attach the declared signatures.  Raises if the
    library was not built: the GPU path never falls back to anything else."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"libwasr_gpu.so not built ({p}); run __graft_entry__.build()")
    lib = C.CDLL(p, mode=C.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def ptr(a) -> int:
    """Raw address of a numpy array or torch tensor (device or host)."""
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data
