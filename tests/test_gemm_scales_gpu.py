"""The tcgen05 GEMMs with block-scale bytes drawn uniformly from every positive
finite e4m3 byte, 0x01..0x7E: subnormal scales and mantissa bits go through
the MMA's unsigned-e4m3 scale read.

Products of two such scales reach 448^2, so the codes are limited to 0 and
+-0.5 (mask 0x99; half of them zeroed for the dual GEMM) to keep most outputs
inside fp16.  The check is scale-invariant and tighter than the contract
tolerance: every output whose exact (float64) value is below 60000 in
magnitude must lie within 1 fp16 ulp plus an fp32-accumulation bound of it,
and every output whose exact value exceeds 66000 must be an infinity of the
same sign.  The dequantised products are exact in fp32 (2 x 2 code bits and
4 x 4 scale bits), so the only arithmetic error is the fp32 sum and the final
rounding.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ACC_REL = 1e-5          # fp32 summation error bound, relative to the sum of |terms| (K <= 512)
FINITE_MAX, INF_MIN = 60000.0, 66000.0


def _ops(pkg, rows_list, K, seed, keep=1.0):
    g = torch.Generator().manual_seed(seed)
    return [pkg.inputs.operand(r, K, g, all_scale_bytes=True, code_mask=0x99, keep=keep) for r in rows_list]


def _deq(oracle, op):
    return oracle.dequant_matrix(op.codes, op.sf_blocked, op.rows, op.K).astype(np.float64)


def _check(got, exact, tol):
    got = got.astype(np.float64)
    fin = np.abs(exact) < FINITE_MAX
    ulp = np.abs(np.spacing(exact[fin].astype(np.float16))).astype(np.float64)
    err = np.abs(got[fin] - exact[fin])
    bad = err > ulp + tol[fin]
    assert not bad.any(), f"{bad.sum()} of {fin.sum()} finite outputs off; worst {np.max(err - ulp - tol[fin])}"
    big = np.abs(exact) > INF_MIN
    assert np.array_equal(np.isinf(got[big]) & (np.sign(got[big]) == np.sign(exact[big])), np.ones(big.sum(), bool))
    assert fin.mean() > 0.5, "test inputs should keep most outputs finite"


def _all_bytes_used(*ops):
    seen = np.zeros(256, bool)
    for op in ops:
        seen[np.unique(op.sf_blocked.cpu().numpy())] = True
    return seen[1:127].all()


@pytest.mark.parametrize("Ms,N,K", [([256, 128], 512, 256), ([200, 64, 333], 384, 512)])
def test_grouped_gemm_all_scale_bytes(pkg, oracle, cuda, Ms, N, K):
    ops = _ops(pkg, Ms + [N] * len(Ms), K, seed=sum(Ms) + K)
    As, Bs = ops[: len(Ms)], ops[len(Ms):]
    assert _all_bytes_used(*ops)
    cs = [torch.full((m, N), float("nan"), dtype=torch.float16, device=cuda) for m in Ms]
    pkg.grouped_gemm([a.codes.to(cuda) for a in As], [b.codes.to(cuda) for b in Bs],
                     [a.sf_blocked.to(cuda) for a in As], [b.sf_blocked.to(cuda) for b in Bs], cs)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    for a, b, c in zip(As, Bs, cs):
        A, B = _deq(oracle, a), _deq(oracle, b)
        _check(c.cpu().numpy(), A @ B.T, ACC_REL * (np.abs(A) @ np.abs(B).T))


def test_dual_gemm_all_scale_bytes(pkg, oracle, cuda):
    M, N, K = 256, 512, 256
    x, w1, w2 = _ops(pkg, [M, N, N], K, seed=17, keep=0.5)
    assert _all_bytes_used(x, w1, w2)
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
    d = lambda t: t.to(cuda)
    pkg.dual_gemm(d(x.codes), d(w1.codes), d(w2.codes), d(x.sf_blocked), d(w1.sf_blocked), d(w2.sf_blocked), c)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    X, W1, W2 = _deq(oracle, x), _deq(oracle, w1), _deq(oracle, w2)
    g, u = X @ W1.T, X @ W2.T
    with np.errstate(over="ignore"):
        silu = g / (1.0 + np.exp(-g))
    exact = silu * u
    # fp32 errors of g and u (summation) propagate through silu(g) * u (|silu'| <= 1.1);
    # the gate itself is evaluated in fp32 with fast exp / divide (relative 1e-5)
    dg = ACC_REL * (np.abs(X) @ np.abs(W1).T)
    du = ACC_REL * (np.abs(X) @ np.abs(W2).T)
    tol = 1.1 * dg * np.abs(u) + np.abs(silu) * du + 1e-5 * np.abs(exact)
    _check(c.cpu().numpy(), exact, tol)


@pytest.mark.parametrize("T,N,K", [(16, 1024, 256), (40, 384, 512)])
def test_skinny_gemm_all_scale_bytes(pkg, oracle, cuda, T, N, K):
    x, w = _ops(pkg, [T, N], K, seed=T + N)
    assert _all_bytes_used(w)
    out = torch.full((T, N), float("nan"), dtype=torch.float16, device=cuda)
    pkg.skinny_gemm(x.codes.to(cuda), w.codes.to(cuda), x.sf_blocked.to(cuda), w.sf_blocked.to(cuda), out)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    X, W = _deq(oracle, x), _deq(oracle, w)
    _check(out.cpu().numpy(), X @ W.T, ACC_REL * (np.abs(X) @ np.abs(W).T))
