"""Shared test setup: the `gpu` marker, and imports of the package (its directory name has
hyphens, so it is registered under the module name ``wechat_asr_gpu_b200``) and of the
CPU oracle (test infrastructure)."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "wechat-asr-gpu_b200")


def load_pkg():
    name = "wechat_asr_gpu_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    if os.path.join(ROOT, "oracle") not in sys.path:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402
    return oracle


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    o = load_oracle()
    o.build()
    return o


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_lib(pkg):
    if not has_gpu():
        pytest.skip("no GPU")
    return pkg.abi.load()


class Dev:
    """Device buffers through the library's own ABI (wp_alloc / wp_h2d / wp_d2h)."""

    def __init__(self, lib):
        self.L = lib
        self.ptrs = []

    def put(self, a):
        a = __import__("numpy").ascontiguousarray(a)
        p = self.L.wp_alloc(max(a.nbytes, 1))
        assert p, "wp_alloc failed"
        self.ptrs.append(p)
        if a.nbytes:
            assert self.L.wp_h2d(p, a.ctypes.data, a.nbytes) == 0
        return p

    def empty(self, nbytes):
        p = self.L.wp_alloc(max(nbytes, 1))
        assert p
        self.ptrs.append(p)
        return p

    def get(self, p, shape, dtype):
        np = __import__("numpy")
        out = np.empty(shape, dtype)
        if out.nbytes:
            assert self.L.wp_d2h(out.ctypes.data, p, out.nbytes) == 0
        return out

    def free(self):
        for p in self.ptrs:
            self.L.wp_free(p)
        self.ptrs = []


@pytest.fixture()
def dev(gpu_lib):
    d = Dev(gpu_lib)
    yield d
    d.free()
