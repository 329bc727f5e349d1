"""NVFP4 block-scaled GEMV: the operator surface of the reference.

``custom_kernel(a, b, scale_a, scale_b, c)`` takes the tensors the reference's
``nvfp4_gemv_forward(a, b, sa, sb, c, M, K, L)`` takes
(blackwell_nvfp4_gemv.cu:500-524) and derives M, K, L from them:

* ``a``       [M, K/2, L]   uint8 or torch.float4_e2m1fn_x2, K contiguous
* ``b``       [>=1, K/2, L] same dtype; row 0 is the vector (:257-259)
* ``scale_a`` [M, K/16, L]  uint8 or torch.float8_e4m3fn
* ``scale_b`` [>=1, K/16, L]
* ``c``       [M, 1, L]     float16, written in place and returned

Unlike the reference, it checks shapes, dtypes, devices and strides, runs on the
current CUDA stream (the reference uses the legacy default stream, :496), and
turns library status codes into ``RuntimeError``.
"""
from __future__ import annotations

import torch

from . import _lib

_FP4_DTYPES = (torch.uint8,) + ((torch.float4_e2m1fn_x2,) if hasattr(torch, "float4_e2m1fn_x2") else ())
_FP8_DTYPES = (torch.uint8, torch.float8_e4m3fn)


def _check3(name: str, t, dtypes) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype not in dtypes:
        raise TypeError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if t.dim() != 3:
        raise ValueError(f"{name} must be 3-D, got shape {tuple(t.shape)}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.shape[1] > 1 and t.stride(1) != 1:
        raise ValueError(f"{name} must be contiguous along its second dimension, strides {t.stride()}")


def gemv_raw(a, b, sfa, sfb, c, M: int, K: int, L: int, stream: int | None = None) -> None:
    """Launch through the C ABI with the strides read from the tensors (no
    checks beyond the library's own)."""
    if stream is None:
        stream = torch.cuda.current_stream(c.device).cuda_stream
    sa, sb, ssa, ssb, sc = a.stride(), b.stride(), sfa.stride(), sfb.stride(), c.stride()
    _lib.check(_lib.lib().nvfp4_gemv(
        a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), c.data_ptr(),
        M, K, L, sa[0], sa[2], sb[2], ssa[0], ssa[2], ssb[2], sc[0], sc[2], stream))


def custom_kernel(a, b=None, scale_a=None, scale_b=None, c=None):
    """c[m, 0, l] = sum_k a[m,k,l] * b[0,k,l] * scale_a[m,k//16,l] * scale_b[0,k//16,l].

    Also accepts a single tuple ``(a, b, scale_a, scale_b, c)``.
    """
    if b is None and isinstance(a, (tuple, list)):
        a, b, scale_a, scale_b, c = a
    _check3("a", a, _FP4_DTYPES)
    _check3("b", b, _FP4_DTYPES)
    _check3("scale_a", scale_a, _FP8_DTYPES)
    _check3("scale_b", scale_b, _FP8_DTYPES)
    if not isinstance(c, torch.Tensor) or c.dtype != torch.float16 or c.dim() != 3:
        raise TypeError("c must be a 3-D float16 tensor [M, 1, L]")
    M, KB, L = a.shape
    K = 2 * KB
    bs, sas, sbs, cs = b.shape, scale_a.shape, scale_b.shape, c.shape
    if bs[1] != KB or bs[2] != L or bs[0] < 1:
        raise ValueError(f"b shape {tuple(bs)} does not match a {tuple(a.shape)}")
    if sas[0] != M or sas[1] * 16 != K or sas[2] != L:
        raise ValueError(f"scale_a shape {tuple(sas)}, expected {(M, K // 16, L)}")
    if sbs[1] * 16 != K or sbs[2] != L or sbs[0] < 1:
        raise ValueError(f"scale_b shape {tuple(sbs)} does not match K={K}, L={L}")
    if cs[0] != M or cs[2] != L:
        raise ValueError(f"c shape {tuple(cs)}, expected {(M, 1, L)}")
    dev = c.device
    if not (a.device == b.device == scale_a.device == scale_b.device == dev):
        raise ValueError("all tensors must be on one device")
    if dev.index != torch.cuda.current_device():
        with torch.cuda.device(dev):
            gemv_raw(a, b, scale_a, scale_b, c, M, K, L)
    else:
        gemv_raw(a, b, scale_a, scale_b, c, M, K, L)
    return c


def nvfp4_gemv_forward(a, b, sa, sb, c, M: int, K: int, L: int) -> None:
    """The reference's own entry point, same name, arguments and in-place
    semantics (blackwell_nvfp4_gemv.cu:500-524): computes the first M rows, K
    elements and L batches of the given tensors into ``c`` and returns None.

    The reference trusts M, K and L; here they must fit inside the tensors
    (ValueError otherwise: larger values would read past them), K must be a
    multiple of 16, and the tensors must be CUDA tensors of the dtypes
    ``custom_kernel`` accepts.  Strides come from the tensors, as in the
    reference.
    """
    M, K, L = int(M), int(K), int(L)
    for name, t in (("a", a), ("b", b), ("sa", sa), ("sb", sb), ("c", c)):
        if not isinstance(t, torch.Tensor) or t.dim() != 3:
            raise TypeError(f"{name} must be a 3-D torch.Tensor")
    if M < 1 or L < 1 or K < 16 or K % 16:
        raise ValueError(f"need M >= 1, L >= 1 and K a positive multiple of 16 (got M={M}, K={K}, L={L})")
    if M > a.shape[0] or K // 2 > a.shape[1] or L > a.shape[2]:
        raise ValueError(f"M={M}, K={K}, L={L} exceed a's shape {tuple(a.shape)}")
    if K // 2 > b.shape[1] or L > b.shape[2]:
        raise ValueError(f"K={K}, L={L} exceed b's shape {tuple(b.shape)}")
    if M > sa.shape[0] or K // 16 > sa.shape[1] or L > sa.shape[2]:
        raise ValueError(f"M={M}, K={K}, L={L} exceed sa's shape {tuple(sa.shape)}")
    if K // 16 > sb.shape[1] or L > sb.shape[2]:
        raise ValueError(f"K={K}, L={L} exceed sb's shape {tuple(sb.shape)}")
    if M > c.shape[0] or L > c.shape[2]:
        raise ValueError(f"M={M}, L={L} exceed c's shape {tuple(c.shape)}")
    if c.dtype != torch.float16:
        raise TypeError("c must be float16")
    _check3("a", a, _FP4_DTYPES)
    _check3("b", b, _FP4_DTYPES)
    _check3("sa", sa, _FP8_DTYPES)
    _check3("sb", sb, _FP8_DTYPES)
    dev = c.device
    if not (a.device == b.device == sa.device == sb.device == dev):
        raise ValueError("all tensors must be on one device")
    with torch.cuda.device(dev):
        gemv_raw(a, b, sa, sb, c, M, K, L)
