"""Fused NVFP4 quantisation of fp16 activations for the GEMMs.

``quantize(x)`` returns ``(codes, scales_blocked)``: e2m1 codes [M, K/2]
(uint8, two per byte, low nibble first) and e4m3 block-16 scales already in
the 128x4 blocked layout that ``dual_gemm`` / ``grouped_gemm`` take.  Rules per
16-element block (global scale 1.0): s = e4m3(amax / 6), q = e2m1(x * fl32(1/s)),
both round-to-nearest-even with saturation; an all-zero block quantises to zeros.
"""
from __future__ import annotations

import torch

from . import _lib
from .layout import blocked_numel


def quantize(x: torch.Tensor, codes: torch.Tensor | None = None, scales: torch.Tensor | None = None):
    if not isinstance(x, torch.Tensor) or x.dtype != torch.float16 or x.dim() != 2 or x.device.type != "cuda":
        raise TypeError("x must be a 2-D float16 CUDA tensor [M, K]")
    if x.stride(1) != 1:
        raise ValueError("x must be contiguous along K")
    M, K = x.shape
    if K % 16:
        raise ValueError("K must be a multiple of 16")
    if codes is None:
        codes = torch.empty((M, K // 2), dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty(blocked_numel(M, K // 16), dtype=torch.uint8, device=x.device)
    if codes.shape != (M, K // 2) or codes.stride(1) != 1 or scales.numel() != blocked_numel(M, K // 16):
        raise ValueError("output buffers have the wrong shape")
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().nvfp4_quantize(x.data_ptr(), M, K, x.stride(0), codes.data_ptr(), codes.stride(0),
                                             scales.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream))
    return codes, scales
