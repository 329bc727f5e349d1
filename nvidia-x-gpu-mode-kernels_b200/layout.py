"""Scale-factor layouts.

The tcgen05 block-scaled MMA reads e4m3 block scales from tensor memory in a
fixed arrangement, and the cheapest way to get them there is a plain copy of a
"128x4 blocked" image from global memory.  A scale matrix S[rows, kb]
(kb = K/16) is cut into tiles of 128 rows x 4 scale columns (= 128 rows x 64 K
elements); tiles are stored row-tile-major, 512 bytes each, and inside a tile
S[r, c] sits at byte ``(r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)``.
Rows pad to a multiple of 128 and kb to a multiple of 4 with zero bytes.

These helpers run on whatever device the input lives on (torch ops only).
"""
from __future__ import annotations

import torch


def blocked_numel(rows: int, kb: int) -> int:
    return ((rows + 127) // 128) * ((kb + 3) // 4) * 512


def to_blocked(s: torch.Tensor) -> torch.Tensor:
    """[rows, kb] uint8/e4m3 -> flat uint8 blocked image."""
    if s.dtype != torch.uint8:
        s = s.view(torch.uint8)
    rows, kb = s.shape
    rp, kp = (rows + 127) // 128 * 128, (kb + 3) // 4 * 4
    if (rp, kp) != (rows, kb):
        z = torch.zeros((rp, kp), dtype=torch.uint8, device=s.device)
        z[:rows, :kb] = s
        s = z
    # [rt, 4(r/32 in tile), 32(r%32), kt, 4(c)] -> [rt, kt, 32, 4, 4]
    t = s.reshape(rp // 128, 4, 32, kp // 4, 4).permute(0, 3, 2, 1, 4)
    return t.contiguous().reshape(-1)


def from_blocked(flat: torch.Tensor, rows: int, kb: int) -> torch.Tensor:
    """Inverse of ``to_blocked`` (drops the padding)."""
    if flat.dtype != torch.uint8:
        flat = flat.view(torch.uint8)
    rp, kp = (rows + 127) // 128 * 128, (kb + 3) // 4 * 4
    t = flat.reshape(rp // 128, kp // 4, 32, 4, 4).permute(0, 3, 2, 1, 4)
    return t.reshape(rp, kp)[:rows, :kb].contiguous()
