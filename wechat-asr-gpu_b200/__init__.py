"""wechat-asr-gpu_b200 -- B200-native (sm_100a) batch-transcription compute layer.

The product is the C-ABI shared library ``libwasr_gpu.so`` (sources in ``csrc/``, headers
in ``include/`` at the repository root): the reference's ``wp_*`` / ``wk_*`` entry points
plus the additive batched engine (``wasr_*``).  This package is the Python host side over
that ABI:

  * :mod:`.abi`    -- ctypes bindings and the weight-blob plan struct
  * :mod:`.synth`  -- seeded synthetic models, audio and workload configurations
  * :mod:`.xnet`   -- the reference's model directory (.xnet + dictionary): parse, load, write
  * :mod:`.stream` -- the reference's streaming front end (Stream::push / partial / finish,
                      src/stream.rs) and text output (Model::text, tidy) over the engine
  * :mod:`.host`   -- ``Engine`` (batched engine) and ``Gpu`` / ``WindowModel``, a mirror of
                      the reference's Rust FFI wrapper (src/gpu.rs) and per-window GPU
                      forward (src/model.rs:504-619) driven through the reference ABI
  * :mod:`.build`  -- in-tree nvcc build for sm_100a

There is no CPU fallback anywhere on this path: if the library is missing, loading fails.
"""
from . import abi, dist, stream, synth, xnet  # noqa: F401
from .host import Engine, Gpu, WindowModel, fbank, ctc_collapse  # noqa: F401

__all__ = ["abi", "dist", "stream", "synth", "xnet", "Engine", "Gpu", "WindowModel", "fbank", "ctc_collapse"]
