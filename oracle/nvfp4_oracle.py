"""CPU oracle for the NVFP4 GEMV / dual GEMM / grouped GEMM path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` may import this module, and only to check or
to time the CPU arm.  The product (the CUDA library and its Python layer)
never calls it and has no CPU fallback.

What it restates
----------------
The reference ships one kernel, ``blackwell_nvfp4_gemv.cu``.  Its arithmetic is

    c[m, 0, l] = sum_k dec_e2m1(A[m, k, l]) * dec_e2m1(b[0, k, l])
                        * dec_e4m3(SFA[m, k//16, l]) * dec_e4m3(SFB[0, k//16, l])

(``fp4_dot``, ``blackwell_nvfp4_gemv.cu:72-139``: e4m3 scale pairs decoded by
``cvt.rn.f16x2.e4m3x2`` at :85-86, e2m1 codes by ``cvt.rn.f16x2.e2m1x2`` at
:94-124, one scale per 16 K-elements, summed over K by the kernel loop
:371-443 and the lane reduction :453-456, stored as fp16 at :458-472).
The reference performs the inner sums in fp16; this oracle follows the
north-star contract instead: dequantise every element to fp32 exactly
(e2m1 x e4m3 is exact in fp32), fp32 matmul, one rounding to fp16.

Tensor layouts follow the reference's tensor-map encoders
(``blackwell_nvfp4_gemv.cu:205-293``):

* A   ``[M, K/2, L]`` bytes, two e2m1 codes per byte, K contiguous;
* b   ``[>=1, K/2, L]`` bytes, only row 0 is read (:257-259);
* SFA ``[M, K/16, L]`` e4m3 bytes;  SFB ``[>=1, K/16, L]`` (:284-286);
* c   ``[M, 1, L]`` fp16.

The e2m1 nibble order inside a byte (low nibble = even K index) does not
change a dot product as long as both operands use the same order, which both
the reference and this oracle do.

The dual GEMM and grouped GEMM have no reference code (the reference README
only announces a dual GEMM).  Their contract is the north-star text: fp32
dequantise-then-matmul, fp16 output, e4m3 block-16 scales stored in the
128x4 blocked ("swizzled") layout that the tcgen05 block-scaled MMA consumes.
Parity for those two is therefore pinned only by this restatement.
"""
from __future__ import annotations

import numpy as np
import torch

# ---------------------------------------------------------------------------
# Element decodes (bit-exact).
# ---------------------------------------------------------------------------

#: e2m1: bit 3 sign, bits 2..1 exponent (bias 1), bit 0 mantissa.  Exponent 0 is
#: subnormal (value m * 0.5).  Values: 0, .5, 1, 1.5, 2, 3, 4, 6 and negatives.
def _e2m1_value(code: int) -> float:
    s = -1.0 if code & 0x8 else 1.0
    e = (code >> 1) & 0x3
    m = code & 0x1
    if e == 0:
        return s * 0.5 * m
    return s * (2.0 ** (e - 1)) * (1.0 + 0.5 * m)


E2M1_LUT = np.array([_e2m1_value(c) for c in range(16)], dtype=np.float32)


def e4m3_value(byte: int) -> float:
    """e4m3fn: bit 7 sign, bits 6..3 exponent (bias 7), bits 2..0 mantissa.
    No infinities; 0x7F and 0xFF are NaN; exponent 0 is subnormal."""
    s = -1.0 if byte & 0x80 else 1.0
    e = (byte >> 3) & 0xF
    m = byte & 0x7
    if e == 0xF and m == 0x7:
        return float("nan")
    if e == 0:
        return s * (m / 8.0) * 2.0 ** -6
    return s * (1.0 + m / 8.0) * 2.0 ** (e - 7)


E4M3_LUT = np.array([e4m3_value(b) for b in range(256)], dtype=np.float32)


def _u8(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu()
        if t.dtype != torch.uint8:
            t = t.view(torch.uint8)
        return t.numpy()
    return np.asarray(t, dtype=np.uint8)


def decode_e2m1(packed) -> np.ndarray:
    """[..., n] bytes -> [..., 2n] float32, low nibble first."""
    p = _u8(packed)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.float32)
    out[..., 0::2] = E2M1_LUT[p & 0xF]
    out[..., 1::2] = E2M1_LUT[p >> 4]
    return out


def decode_e4m3(scales) -> np.ndarray:
    return E4M3_LUT[_u8(scales)]


# ---------------------------------------------------------------------------
# 128x4 blocked scale layout (the layout tcgen05 block-scaled MMA reads).
# A scale matrix S[rows, kb] (kb = K/16) is cut into 128-row x 4-column tiles;
# tiles are stored row-tile-major (all K tiles of row tile 0 first), 512 bytes
# each; inside a tile, S[r, c] sits at byte (r % 32) * 16 + (r // 32) * 4 + c.
# Rows are padded to a multiple of 128 and kb to a multiple of 4 with zeros.
# ---------------------------------------------------------------------------

def blocked_size(rows: int, kb: int) -> int:
    return ((rows + 127) // 128) * ((kb + 3) // 4) * 512


def to_blocked_ref(s: np.ndarray) -> np.ndarray:
    """Plain [rows, kb] scale bytes -> flat blocked bytes (pure index loops)."""
    s = _u8(s)
    rows, kb = s.shape
    nrt, nkt = (rows + 127) // 128, (kb + 3) // 4
    out = np.zeros(nrt * nkt * 512, dtype=np.uint8)
    r = np.arange(rows)[:, None]
    c = np.arange(kb)[None, :]
    off = ((r // 128) * nkt + (c // 4)) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)
    out[off] = s
    return out


def from_blocked_ref(flat, rows: int, kb: int) -> np.ndarray:
    flat = _u8(flat).reshape(-1)
    nkt = (kb + 3) // 4
    r = np.arange(rows)[:, None]
    c = np.arange(kb)[None, :]
    off = ((r // 128) * nkt + (c // 4)) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)
    return flat[off]


# ---------------------------------------------------------------------------
# GEMV (the reference's path).
# ---------------------------------------------------------------------------

def _dequant_rows(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """codes [R, K/2] bytes, scales [R, K/16] e4m3 bytes -> [R, K] fp32."""
    v = decode_e2m1(codes)
    sf = decode_e4m3(scales)
    return (v.reshape(v.shape[0], -1, 16) * sf[:, :, None]).reshape(v.shape[0], -1)


def gemv(a, b, sfa, sfb, M: int, K: int, L: int, acc=np.float32) -> np.ndarray:
    """Returns c as a float16 array [M, 1, L] (acc=np.float64 keeps the result
    unrounded, as a float64 array, for ulp-level checks)."""
    a, b, sfa, sfb = _u8(a), _u8(b), _u8(sfa), _u8(sfb)
    out = np.empty((M, 1, L), dtype=np.float16 if acc == np.float32 else np.float64)
    for l in range(L):
        A = _dequant_rows(a[:M, : K // 2, l], sfa[:M, : K // 16, l]).astype(acc)
        bv = _dequant_rows(b[:1, : K // 2, l], sfb[:1, : K // 16, l])[0].astype(acc)
        r = A @ bv
        with np.errstate(over="ignore"):   # beyond fp16 range the output is inf, as on the GPU
            out[:, 0, l] = r.astype(np.float16) if acc == np.float32 else r
    return out


def gemv_torch(a, b, sfa, sfb, M: int, K: int, L: int) -> torch.Tensor:
    """The same restatement with torch CPU ops (multi-threaded); this is the
    timed CPU baseline.  Decode: 16-entry LUT for e2m1 (torch cannot cast fp4
    on the CPU) and a 256-entry LUT for e4m3, both built from the bit formulas
    above; fp32 matmul; fp16 output [M, 1, L]."""
    lut2 = torch.from_numpy(E2M1_LUT)
    lut8 = torch.from_numpy(E4M3_LUT)
    a = a.view(torch.uint8) if a.dtype != torch.uint8 else a
    b = b.view(torch.uint8) if b.dtype != torch.uint8 else b
    sfa = sfa.view(torch.uint8) if sfa.dtype != torch.uint8 else sfa
    sfb = sfb.view(torch.uint8) if sfb.dtype != torch.uint8 else sfb
    out = torch.empty((M, 1, L), dtype=torch.float16)
    for l in range(L):
        ab = a[:M, : K // 2, l].long()
        A = torch.stack((lut2[ab & 15], lut2[ab >> 4]), dim=-1).reshape(M, K)
        A = (A.view(M, K // 16, 16) * lut8[sfa[:M, : K // 16, l].long()][:, :, None]).view(M, K)
        bb = b[0, : K // 2, l].long()
        bv = torch.stack((lut2[bb & 15], lut2[bb >> 4]), dim=-1).reshape(K)
        bv = (bv.view(K // 16, 16) * lut8[sfb[0, : K // 16, l].long()][:, None]).view(K)
        out[:, 0, l] = (A @ bv).to(torch.float16)
    return out


# ---------------------------------------------------------------------------
# GEMMs (no reference code; contract from the north star).
# ---------------------------------------------------------------------------

def dequant_matrix(codes, sf_blocked, rows: int, K: int) -> np.ndarray:
    """codes [rows, K/2] bytes + blocked scales -> [rows, K] fp32."""
    s = from_blocked_ref(sf_blocked, rows, K // 16)
    return _dequant_rows(_u8(codes)[:rows, : K // 2], s)


def gemm(a, b, sfa_blocked, sfb_blocked, M: int, N: int, K: int, acc=np.float32) -> np.ndarray:
    """C[M, N] = A[M, K] . B[N, K]^T, both K-major e2m1 with blocked scales."""
    A = dequant_matrix(a, sfa_blocked, M, K).astype(acc)
    B = dequant_matrix(b, sfb_blocked, N, K).astype(acc)
    return A @ B.T


def silu(x):
    return x / (1.0 + np.exp(-x))


def dual_gemm(x, w1, w2, sfx, sfw1, sfw2, M: int, N: int, K: int, acc=np.float32) -> np.ndarray:
    """out[M, N] = silu(X W1^T) * (X W2^T) computed in fp32 (or acc), fp16 out
    when acc is fp32."""
    X = dequant_matrix(x, sfx, M, K).astype(acc)
    g = X @ dequant_matrix(w1, sfw1, N, K).astype(acc).T
    u = X @ dequant_matrix(w2, sfw2, N, K).astype(acc).T
    r = silu(g) * u
    return r.astype(np.float16) if acc == np.float32 else r


def grouped_gemm(groups, acc=np.float32):
    """groups: iterable of (a, b, sfa_blocked, sfb_blocked, M, N, K)."""
    outs = []
    for a, b, sfa, sfb, M, N, K in groups:
        r = gemm(a, b, sfa, sfb, M, N, K, acc)
        outs.append(r.astype(np.float16) if acc == np.float32 else r)
    return outs


def dequant_matrix_torch(codes, sf_blocked, rows: int, K: int) -> torch.Tensor:
    """torch CPU form of ``dequant_matrix`` (multi-threaded; the timed CPU
    baseline of the GEMMs): codes [rows, K/2] bytes + blocked scales ->
    [rows, K] fp32, via the same 16- and 256-entry decode tables."""
    lut2 = torch.from_numpy(E2M1_LUT)
    lut8 = torch.from_numpy(E4M3_LUT)
    c = codes if codes.dtype == torch.uint8 else codes.view(torch.uint8)
    c = c[:rows, : K // 2].long()
    v = torch.stack((lut2[c & 15], lut2[c >> 4]), dim=-1).reshape(rows, K)
    s = torch.from_numpy(from_blocked_ref(sf_blocked, rows, K // 16).astype(np.int64))
    return (v.view(rows, K // 16, 16) * lut8[s][:, :, None]).view(rows, K)


def gemm_torch(a, b, sfa_blocked, sfb_blocked, M: int, N: int, K: int) -> torch.Tensor:
    """``gemm`` with torch CPU ops: fp32 C[M, N] (no reference code exists)."""
    return dequant_matrix_torch(a, sfa_blocked, M, K) @ dequant_matrix_torch(b, sfb_blocked, N, K).T


def dual_gemm_torch(x, w1, w2, sfx, sfw1, sfw2, M: int, N: int, K: int) -> torch.Tensor:
    """``dual_gemm`` with torch CPU ops: fp16 silu(X W1^T) * (X W2^T)."""
    X = dequant_matrix_torch(x, sfx, M, K)
    g = X @ dequant_matrix_torch(w1, sfw1, N, K).T
    u = X @ dequant_matrix_torch(w2, sfw2, N, K).T
    return (torch.nn.functional.silu(g) * u).to(torch.float16)


# ---------------------------------------------------------------------------
# Quantiser (north-star "next" row: fp16 activations -> NVFP4).  No reference
# code exists; these are the rounding rules the library documents.
# ---------------------------------------------------------------------------

def _round_half_even(v: np.ndarray) -> np.ndarray:
    return np.round(v)   # numpy rounds halves to even


def e4m3_rne_satfinite(v: np.ndarray) -> np.ndarray:
    """Non-negative float64 -> e4m3fn byte, round-to-nearest-even, saturating
    at 448 (the largest finite value)."""
    v = np.asarray(v, dtype=np.float64)
    out = np.zeros(v.shape, dtype=np.uint8)
    pos = v > 0
    e = np.floor(np.log2(np.where(pos, v, 1.0)))
    e = np.clip(e, -6, 8)                                   # subnormals share the 2^-6 binade's spacing
    spacing = 2.0 ** (e - 3)
    q = _round_half_even(v / spacing) * spacing              # may step into the next binade: still exact
    q = np.minimum(q, 448.0)
    # encode q
    qe = np.floor(np.log2(np.where(q > 0, q, 1.0)))
    normal = q >= 2.0 ** -6
    exp_field = np.where(normal, qe + 7, 0).astype(np.int64)
    mant = np.where(normal, q / 2.0 ** qe - 1.0, q / 2.0 ** -6) * 8
    code = (exp_field << 3) | np.round(mant).astype(np.int64)
    out[pos] = code[pos].astype(np.uint8)
    return out


_E2M1_POS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_rne_satfinite(v: np.ndarray) -> np.ndarray:
    """float -> e2m1 code (sign bit 3), round-to-nearest-even, |v| > 6 -> 6."""
    v = np.asarray(v, dtype=np.float64)
    a = np.minimum(np.abs(v), 6.0)
    idx = np.searchsorted(_E2M1_POS, a)                      # first grid point >= a
    idx = np.clip(idx, 1, 7)
    lo, hi = _E2M1_POS[idx - 1], _E2M1_POS[idx]
    mag = np.where(a - lo < hi - a, idx - 1, np.where(a - lo > hi - a, idx, np.where((idx - 1) % 2 == 0, idx - 1, idx)))
    mag = np.where(a == 0, 0, mag)
    return (mag | np.where(np.signbit(v), 8, 0)).astype(np.uint8)


def quantize(x) -> tuple[np.ndarray, np.ndarray]:
    """x [M, K] fp16 -> (codes [M, K/2] uint8, blocked scale bytes)."""
    x = np.asarray(x, dtype=np.float16).astype(np.float32)
    M, K = x.shape
    blocks = x.reshape(M, K // 16, 16)
    amax = np.abs(blocks).max(axis=2)
    sbyte = e4m3_rne_satfinite((amax / np.float32(6.0)).astype(np.float32).astype(np.float64))
    s = E4M3_LUT[sbyte].astype(np.float32)
    safe = np.where(s > 0, s, np.float32(1.0))
    inv = (np.float32(1.0) / safe).astype(np.float32)        # one IEEE f32 division per block
    qv = (blocks * inv[:, :, None]).astype(np.float32)       # f32 product, correctly rounded
    codes = e2m1_rne_satfinite(qv.astype(np.float64))
    codes = np.where((s > 0)[:, :, None], codes, 0).astype(np.uint8).reshape(M, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, to_blocked_ref(sbyte)
