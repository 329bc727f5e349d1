"""NVFP4 dual GEMM (fused SiLU gate) and grouped GEMM on the tcgen05 tensor cores.

No reference code exists for either (the reference ships only the GEMV and
announces a dual GEMM, README.md:3); the operator surface mirrors the GEMV's
``custom_kernel``: caller-owned tensors, the output written in place and
returned, RuntimeError on a library error.

Operand conventions (see include/nvfp4_b200.h):

* codes: ``[rows, K/2]`` uint8 or ``torch.float4_e2m1fn_x2``, K contiguous;
* scales: e4m3 bytes (uint8 or ``torch.float8_e4m3fn``), non-negative, either
  already in the 128x4 blocked layout (any shape, ``layout.blocked_numel``
  elements, contiguous) or plain ``[rows, K/16]`` (converted here with
  ``layout.to_blocked``, which costs extra launches);
* outputs: fp16 ``[M, N]`` with unit column stride.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .layout import blocked_numel, to_blocked

_FP4 = (torch.uint8,) + ((torch.float4_e2m1fn_x2,) if hasattr(torch, "float4_e2m1fn_x2") else ())
_FP8 = (torch.uint8, torch.float8_e4m3fn)


def _codes(name, t, rows=None):
    if not isinstance(t, torch.Tensor) or t.dtype not in _FP4 or t.dim() != 2:
        raise TypeError(f"{name} must be a 2-D uint8 / float4_e2m1fn_x2 tensor [rows, K/2]")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.stride(1) != 1:
        raise ValueError(f"{name} must be contiguous along K")
    if rows is not None and t.shape[0] != rows:
        raise ValueError(f"{name} has {t.shape[0]} rows, expected {rows}")
    return t


def _scales(name, s, rows, K):
    if not isinstance(s, torch.Tensor) or s.dtype not in _FP8:
        raise TypeError(f"{name} must be a uint8 / float8_e4m3fn tensor")
    if s.dim() == 2 and tuple(s.shape) == (rows, K // 16):
        return to_blocked(s)
    if s.numel() != blocked_numel(rows, K // 16) or not s.is_contiguous():
        raise ValueError(f"{name}: expected plain [{rows}, {K // 16}] or a contiguous blocked buffer of "
                         f"{blocked_numel(rows, K // 16)} bytes, got shape {tuple(s.shape)}")
    return s


def _out(c, M, N):
    if not isinstance(c, torch.Tensor) or c.dtype != torch.float16 or tuple(c.shape) != (M, N) or c.stride(1) != 1:
        raise ValueError(f"output must be a float16 [{M}, {N}] tensor with unit column stride")
    return c


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def dual_gemm(a, b1, b2, scale_a, scale_b1, scale_b2, c):
    """c = silu(a . b1^T) * (a . b2^T); a [M, K/2], b1/b2 [N, K/2]."""
    _codes("a", a)
    M, K = a.shape[0], a.shape[1] * 2
    _codes("b1", b1)
    N = b1.shape[0]
    _codes("b2", b2, N)
    if b1.shape[1] * 2 != K or b2.shape[1] * 2 != K or b1.stride(0) != b2.stride(0):
        raise ValueError("b1 and b2 must have the same shape and row stride as each other, and K of a")
    sa = _scales("scale_a", scale_a, M, K)
    s1 = _scales("scale_b1", scale_b1, N, K)
    s2 = _scales("scale_b2", scale_b2, N, K)
    _out(c, M, N)
    with torch.cuda.device(c.device):
        _lib.check(_lib.lib().nvfp4_dual_gemm(
            a.data_ptr(), b1.data_ptr(), b2.data_ptr(), sa.data_ptr(), s1.data_ptr(), s2.data_ptr(), c.data_ptr(),
            M, N, K, a.stride(0), b1.stride(0), c.stride(0), _stream(c.device)))
    return c


def grouped_gemm(a_list, b_list, scale_a_list, scale_b_list, c_list):
    """c_g = a_g . b_g^T for every group g (one persistent launch for up to 24 groups)."""
    G = len(a_list)
    if not (len(b_list) == len(scale_a_list) == len(scale_b_list) == len(c_list) == G) or G == 0:
        raise ValueError("grouped_gemm: all lists must have the same, non-zero length")
    arr = (_lib.Group * G)()
    keep = []
    dev = c_list[0].device
    for i in range(G):
        a, b, c = _codes(f"a[{i}]", a_list[i]), _codes(f"b[{i}]", b_list[i]), c_list[i]
        M, K, N = a.shape[0], a.shape[1] * 2, b.shape[0]
        if M == 0:   # empty group: the library skips it
            arr[i] = _lib.Group(None, None, None, None, None, 0, N, K, 0, 0, 0)
            continue
        if b.shape[1] * 2 != K:
            raise ValueError(f"group {i}: a and b disagree on K")
        sa = _scales(f"scale_a[{i}]", scale_a_list[i], M, K)
        sb = _scales(f"scale_b[{i}]", scale_b_list[i], N, K)
        _out(c, M, N)
        keep += [sa, sb]
        arr[i] = _lib.Group(a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(), c.data_ptr(),
                            M, N, K, a.stride(0), b.stride(0), c.stride(0))
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().nvfp4_grouped_gemm(arr, G, _stream(dev)))
    return c_list


def skinny_gemm(x, w, scale_x, scale_w, out):
    """out[T, N] = x[T, K] . w[N, K]^T for a decode batch of 1 <= T <= 64 token
    rows; the weights stream through the tensor cores as the 128-row MMA
    operand."""
    _codes("x", x)
    T, K = x.shape[0], x.shape[1] * 2
    _codes("w", w)
    N = w.shape[0]
    if w.shape[1] * 2 != K:
        raise ValueError("x and w disagree on K")
    if not 1 <= T <= 64:
        raise ValueError("skinny_gemm takes 1..64 token rows; use grouped_gemm for more")
    sx = _scales("scale_x", scale_x, T, K)
    sw = _scales("scale_w", scale_w, N, K)
    _out(out, T, N)
    with torch.cuda.device(out.device):
        _lib.check(_lib.lib().nvfp4_gemm_skinny(x.data_ptr(), w.data_ptr(), sx.data_ptr(), sw.data_ptr(),
                                                out.data_ptr(), T, N, K, x.stride(0), w.stride(0), out.stride(0),
                                                _stream(out.device)))
    return out
