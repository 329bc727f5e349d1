"""Seeded synthetic inputs for the benchmark configurations.

There is no public dataset for this path; inputs follow the configured
distributions: e2m1 code bytes uniform over 0..255 (so both nibbles are
uniform over all 16 codes) and e4m3 block scales equal to 2^u with u uniform
in [-3, 3], i.e. bytes ``(u + 7) << 3``.  Generation uses a CPU
``torch.Generator`` so the same seed gives the same bytes on every machine;
tensors are then moved to ``device``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .layout import to_blocked


def _codes(g: torch.Generator, shape) -> torch.Tensor:
    return torch.randint(0, 256, shape, dtype=torch.uint8, generator=g)


def _scales(g: torch.Generator, shape, lo: int = -3, hi: int = 3) -> torch.Tensor:
    u = torch.randint(lo, hi + 1, shape, dtype=torch.int16, generator=g)
    return ((u + 7) << 3).to(torch.uint8)


@dataclass
class GemvInputs:
    a: torch.Tensor        # [M, K/2, L] uint8
    b: torch.Tensor        # [1, K/2, L] uint8
    sfa: torch.Tensor      # [M, K/16, L] uint8 (e4m3 bytes)
    sfb: torch.Tensor      # [1, K/16, L]
    c: torch.Tensor        # [M, 1, L] fp16
    M: int
    K: int
    L: int

    def as_tuple(self):
        return self.a, self.b, self.sfa, self.sfb, self.c

    def nbytes_algorithmic(self) -> int:
        M, K, L = self.M, self.K, self.L
        return M * K // 2 * L + M * K // 16 * L + K // 2 * L + K // 16 * L + 2 * M * L


def gemv_inputs(M: int, K: int, L: int, seed: int = 0, device="cpu") -> GemvInputs:
    """Layout as the reference's tensor maps expect (K innermost, L outermost)."""
    g = torch.Generator().manual_seed(seed)
    a = _codes(g, (L, M, K // 2)).permute(1, 2, 0)
    b = _codes(g, (L, 1, K // 2)).permute(1, 2, 0)
    sfa = _scales(g, (L, M, K // 16)).permute(1, 2, 0)
    sfb = _scales(g, (L, 1, K // 16)).permute(1, 2, 0)
    dev = torch.device(device)

    def mv(t):
        # keep the permuted strides when moving
        return t.permute(2, 0, 1).contiguous().to(dev).permute(1, 2, 0)

    c = torch.empty((L, 1, M), dtype=torch.float16, device=dev).permute(2, 1, 0)
    return GemvInputs(mv(a), mv(b), mv(sfa), mv(sfb), c, M, K, L)


@dataclass
class Operand:
    """One K-major NVFP4 matrix: codes [rows, K/2] and blocked scales."""
    codes: torch.Tensor
    sf_blocked: torch.Tensor
    rows: int
    K: int


#: GEMM scale exponents.  The GEMM configurations fix no scale range; with the
#: GEMV's 2^[-3, 3] a K=4096 dual GEMM gives silu(g)*u around 4e7, far beyond
#: fp16, so GEMM operands use 2^u with u in [-5, -3] (outputs of order 1-100).
GEMM_SCALE_EXP = (-5, -3)


def operand(rows: int, K: int, g: torch.Generator, device="cpu", scale_exp=GEMM_SCALE_EXP,
            all_scale_bytes: bool = False, code_mask: int = 0xFF, keep: float = 1.0) -> Operand:
    """Seeded operand.  Scales are 2^u, u uniform in ``scale_exp``, or, with
    ``all_scale_bytes``, uniform over every positive finite e4m3 byte
    0x01..0x7E (subnormals and mantissa bits included).  ``code_mask`` ANDs
    every code byte (0x99 keeps the values 0 and +-0.5, which keeps products of
    large scales inside fp16) and ``keep`` zeroes each code byte with
    probability 1 - keep."""
    codes = _codes(g, (rows, K // 2)) & code_mask
    if keep < 1.0:
        codes = torch.where(torch.rand((rows, K // 2), generator=g) < keep, codes, torch.zeros_like(codes))
    if all_scale_bytes:
        sf = torch.randint(1, 127, (rows, K // 16), dtype=torch.uint8, generator=g)
    else:
        sf = _scales(g, (rows, K // 16), *scale_exp)
    return Operand(codes.to(device), to_blocked(sf).to(device), rows, K)


def grouped_m_sizes(G: int = 8, seed: int = 0, lo: int = 64, hi: int = 1024, step: int = 64) -> list[int]:
    """Per-group M uniform in [lo, hi] in steps of `step`, from the seed."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(lo // step, hi // step + 1, (G,), generator=g) * step).tolist()
