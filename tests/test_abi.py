"""The C-ABI library loads and exports every function include/vq2_b200.h declares; the ctypes
binding declares a signature for each. Host-only calls (no GPU needed): version, strerror."""
import ctypes
import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "vq2_b200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vq2_[a-z0-9_]+)\s*\(", text)))


def _library():
    from vq2_vllm import _lib
    if not os.path.exists(_lib.LIB_PATH):        # build it here (nvcc cross-compiles without a GPU)
        import runpy
        runpy.run_path(os.path.join(REPO, "deepseek-v4-flash-2bit-gb10_b200", "build_lib.py"), run_name="__main__")
    return _lib, ctypes.CDLL(_lib.LIB_PATH)


def test_every_declared_symbol_is_exported():
    _, L = _library()
    names = declared()
    assert len(names) >= 19
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    _lib, _ = _library()
    assert set(declared()) <= set(_lib._SIGS), sorted(set(declared()) - set(_lib._SIGS))


def test_host_only_calls():
    _lib, _ = _library()
    L = _lib.lib()
    assert L.vq2_version() > 0
    assert L.vq2_strerror(0) and L.vq2_strerror(8)
