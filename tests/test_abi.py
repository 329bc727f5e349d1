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


def test_gemm_entry_points_reject_bad_arguments_without_gpu(pkg):
    """Every GEMM-side entry point validates its arguments before any CUDA call."""
    l = pkg._lib.lib()
    msg = lambda: l.nvfp4_last_error()
    p = 4096   # a 16-byte-aligned stand-in address: validation never dereferences it
    # skinny GEMM: token count, K granularity, null operand
    assert l.nvfp4_gemm_skinny(p, p, p, p, p, 0, 128, 256, 128, 128, 128, None) == 1 and b"1..64" in msg()
    assert l.nvfp4_gemm_skinny(p, p, p, p, p, 65, 128, 256, 128, 128, 128, None) == 1 and b"1..64" in msg()
    assert l.nvfp4_gemm_skinny(p, p, p, p, p, 8, 128, 96, 48, 48, 128, None) == 1 and b"multiple of 64" in msg()
    assert l.nvfp4_gemm_skinny(None, p, p, p, p, 8, 128, 256, 128, 128, 128, None) == 1 and b"null" in msg()
    # dual GEMM: K granularity, row stride below K/2, misaligned operand
    assert l.nvfp4_dual_gemm(p, p, p, p, p, p, p, 128, 128, 100, 64, 64, 128, None) == 1
    assert l.nvfp4_dual_gemm(p, p, p, p, p, p, p, 128, 128, 256, 64, 128, 128, None) == 1 and b"stride" in msg()
    assert l.nvfp4_dual_gemm(p + 8, p, p, p, p, p, p, 128, 128, 256, 128, 128, 128, None) == 2
    # grouped GEMM: no groups
    assert l.nvfp4_grouped_gemm(None, 0, None) == 1 and b"no groups" in msg()
    # quantiser: K granularity, odd fp16 address, misaligned scale buffer
    assert l.nvfp4_quantize(p, 8, 24, 24, p, 12, p, None) == 1
    assert l.nvfp4_quantize(p + 1, 8, 32, 32, p, 16, p, None) == 2
    assert l.nvfp4_quantize(p, 8, 32, 32, p, 16, p + 2, None) == 2 and b"4-byte" in msg()
    # tensor-core probe: iteration count and pattern
    assert l.nvfp4_mma_peak_pattern(0, 0, None) == 1
    assert l.nvfp4_mma_peak_pattern(16, 7, None) == 1 and b"pattern" in msg()


def test_allgather_rejects_bad_world_without_gpu(pkg):
    l = pkg._lib.lib()
    stages = (ctypes.c_void_p * 8)(*([4096] * 8))
    # a, b, sfa, sfb, M_local, K, L, strides (6), out, c_sm, c_sl, m_off, M_total, stages, world, rank, epoch, stream
    args = lambda world, rank: (4096, 4096, 4096, 4096, 64, 512, 1, 256, 0, 0, 32, 0, 0,
                                4096, 1, 0, 0, 128, stages, world, rank, 1, None)
    assert l.nvfp4_gemv_allgather(*args(9, 0)) == 1 and b"world" in l.nvfp4_last_error()
    assert l.nvfp4_gemv_allgather(*args(2, 2)) == 1
    nulls = (ctypes.c_void_p * 8)()
    a = list(args(2, 0))
    a[18] = nulls
    assert l.nvfp4_gemv_allgather(*a) == 1 and b"null staging" in l.nvfp4_last_error()
    odd = (ctypes.c_void_p * 8)(*([4100] * 8))
    a[18] = odd
    assert l.nvfp4_gemv_allgather(*a) == 2 and b"8-byte" in l.nvfp4_last_error()
    a = list(args(2, 0))
    a[17] = 32                                  # M_total below m_off + M_local
    assert l.nvfp4_gemv_allgather(*a) == 1 and b"shape" in l.nvfp4_last_error()
    a = list(args(2, 0))
    a[4] = 63                                   # odd share of an even M_total: two results per line
    assert l.nvfp4_gemv_allgather(*a) == 1 and b"even" in l.nvfp4_last_error()


def test_gemv_forward_checks_sizes_against_tensors(pkg):
    """nvfp4_gemv_forward (the reference's binding signature) refuses M, K, L
    that do not fit the tensors before touching any device."""
    import torch
    a = torch.zeros((64, 256, 1), dtype=torch.uint8)
    b = torch.zeros((1, 256, 1), dtype=torch.uint8)
    sa = torch.zeros((64, 32, 1), dtype=torch.uint8)
    sb = torch.zeros((1, 32, 1), dtype=torch.uint8)
    c = torch.zeros((64, 1, 1), dtype=torch.float16)
    with pytest.raises(ValueError, match="exceed a"):
        pkg.nvfp4_gemv_forward(a, b, sa, sb, c, 65, 512, 1)
    with pytest.raises(ValueError, match="exceed a"):
        pkg.nvfp4_gemv_forward(a, b, sa, sb, c, 64, 1024, 1)
    with pytest.raises(ValueError, match="multiple of 16"):
        pkg.nvfp4_gemv_forward(a, b, sa, sb, c, 64, 40, 1)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.nvfp4_gemv_forward(a, b, sa, sb, c, 64, 512, 1)
