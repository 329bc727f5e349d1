"""CPU checks of the C ABI: the library loads without a GPU and exports every
entry point declared in include/*.h; the Python binding declares them all."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(nvfp4_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "nvfp4_gemv" in syms and "nvfp4_last_error" in syms


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports(pkg, name):
    lib = ctypes.CDLL(pkg._lib.LIB_PATH)
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_binding_covers_header(pkg):
    bound = set(pkg._lib.SIGNATURES) | {"nvfp4_last_error"}
    assert set(declared_symbols()) <= bound


def test_version_and_message(pkg):
    l = pkg._lib.lib()
    assert l.nvfp4_version() >= 100
    assert isinstance(l.nvfp4_last_error(), bytes)


def test_gemv_rejects_bad_shapes_without_gpu(pkg):
    """Argument validation happens before any CUDA call."""
    l = pkg._lib.lib()
    rc = l.nvfp4_gemv(1, 1, 1, 1, 1, 4, 24, 1, 12, 0, 0, 2, 0, 0, 1, 0, None)
    assert rc == 1 and b"K%16" in l.nvfp4_last_error()
    rc = l.nvfp4_gemv(None, 1, 1, 1, 1, 4, 32, 1, 16, 0, 0, 2, 0, 0, 1, 0, None)
    assert rc == 1 and b"null" in l.nvfp4_last_error()
    with pytest.raises(RuntimeError, match="INVALID"):
        pkg._lib.check(rc)
