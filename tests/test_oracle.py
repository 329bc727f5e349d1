"""CPU tests of the oracle itself: element decodes, the blocked scale layout,
and the GEMV / GEMM restatements against float64 arithmetic."""
import math

import numpy as np
import pytest
import torch


def test_e2m1_table(oracle):
    expect = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert oracle.E2M1_LUT[:8].tolist() == expect
    assert oracle.E2M1_LUT[8:].tolist() == [-v for v in expect]
    # code 0x8 is negative zero
    assert math.copysign(1.0, float(oracle.E2M1_LUT[8])) == -1.0


def test_e4m3_table_matches_torch(oracle):
    ref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    ours = oracle.E4M3_LUT
    nan = np.isnan(ref)
    assert (np.isnan(ours) == nan).all()
    assert nan.sum() == 2 and nan[0x7F] and nan[0xFF]
    np.testing.assert_array_equal(ours[~nan], ref[~nan])
    # the generator's scale bytes are exact powers of two
    for u in range(-3, 4):
        assert oracle.e4m3_value((u + 7) << 3) == 2.0 ** u
    assert oracle.e4m3_value(0x7E) == 448.0


def test_nibble_order(oracle):
    v = oracle.decode_e2m1(np.array([[0x72]], dtype=np.uint8))
    assert v.tolist() == [[1.0, 6.0]]


@pytest.mark.parametrize("rows,kb", [(128, 4), (256, 256), (7, 3), (130, 9), (1, 1)])
def test_blocked_layout_roundtrip(pkg, oracle, rows, kb):
    g = torch.Generator().manual_seed(rows * 1000 + kb)
    s = torch.randint(0, 256, (rows, kb), dtype=torch.uint8, generator=g)
    ours = pkg.layout.to_blocked(s)
    ref = oracle.to_blocked_ref(s.numpy())
    assert ours.numel() == oracle.blocked_size(rows, kb) == pkg.layout.blocked_numel(rows, kb)
    np.testing.assert_array_equal(ours.numpy(), ref)
    np.testing.assert_array_equal(pkg.layout.from_blocked(ours, rows, kb).numpy(), s.numpy())
    np.testing.assert_array_equal(oracle.from_blocked_ref(ref, rows, kb), s.numpy())


def test_blocked_layout_positions(oracle):
    s = np.zeros((256, 8), dtype=np.uint8)
    s[33, 5] = 7     # row tile 0, k tile 1: (33%32)*16 + (33//32)*4 + 1 = 21
    s[130, 2] = 9    # row tile 1, k tile 0: tile index 2 -> 1024 + 2*16 + 0*4 + 2
    flat = oracle.to_blocked_ref(s)
    assert flat[512 + 21] == 7
    assert flat[2 * 512 + 34] == 9
    assert flat.sum() == 16


def _gemv_f64(oracle, x):
    return oracle.gemv(x.a, x.b, x.sfa, x.sfb, x.M, x.K, x.L, acc=np.float64)


@pytest.mark.parametrize("M,K,L", [(256, 1024, 1), (40, 256, 3), (5, 48, 2)])
def test_gemv_oracle_vs_f64(pkg, oracle, M, K, L):
    x = pkg.inputs.gemv_inputs(M, K, L, seed=1)
    got = oracle.gemv(x.a, x.b, x.sfa, x.sfb, M, K, L).astype(np.float64)
    ref = _gemv_f64(oracle, x)
    np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-3)
    tgot = oracle.gemv_torch(x.a, x.b, x.sfa, x.sfb, M, K, L).numpy().astype(np.float64)
    np.testing.assert_allclose(tgot, ref, rtol=1e-3, atol=1e-3)


def test_gemv_oracle_pure_loops(pkg, oracle):
    """The vectorised restatement against a scalar loop of the formula."""
    M, K, L = 3, 64, 2
    x = pkg.inputs.gemv_inputs(M, K, L, seed=5)
    a, b, sa, sb = (t.numpy() for t in (x.a, x.b, x.sfa, x.sfb))
    got = oracle.gemv(x.a, x.b, x.sfa, x.sfb, M, K, L, acc=np.float64)
    for l in range(L):
        for m in range(M):
            acc = 0.0
            for k in range(K):
                byte_a, byte_b = a[m, k // 2, l], b[0, k // 2, l]
                ca = (byte_a >> 4) if k & 1 else (byte_a & 15)
                cb = (byte_b >> 4) if k & 1 else (byte_b & 15)
                acc += (oracle.E2M1_LUT[ca] * oracle.E2M1_LUT[cb]
                        * oracle.e4m3_value(int(sa[m, k // 16, l])) * oracle.e4m3_value(int(sb[0, k // 16, l])))
            assert got[m, 0, l] == pytest.approx(acc, rel=1e-12, abs=1e-12)


def test_gemm_oracles(pkg, oracle):
    g = torch.Generator().manual_seed(3)
    M, N, K = 70, 130, 128
    x = pkg.inputs.operand(M, K, g)
    w1 = pkg.inputs.operand(N, K, g)
    w2 = pkg.inputs.operand(N, K, g)
    c = oracle.gemm(x.codes, w1.codes, x.sf_blocked, w1.sf_blocked, M, N, K, acc=np.float64)
    X = oracle.decode_e2m1(x.codes.numpy()).reshape(M, K // 16, 16) * oracle.decode_e4m3(
        pkg.layout.from_blocked(x.sf_blocked, M, K // 16).numpy())[:, :, None]
    W = oracle.decode_e2m1(w1.codes.numpy()).reshape(N, K // 16, 16) * oracle.decode_e4m3(
        pkg.layout.from_blocked(w1.sf_blocked, N, K // 16).numpy())[:, :, None]
    np.testing.assert_allclose(c, X.reshape(M, K).astype(np.float64) @ W.reshape(N, K).astype(np.float64).T,
                               rtol=1e-12)
    d = oracle.dual_gemm(x.codes, w1.codes, w2.codes, x.sf_blocked, w1.sf_blocked, w2.sf_blocked, M, N, K)
    d64 = oracle.dual_gemm(x.codes, w1.codes, w2.codes, x.sf_blocked, w1.sf_blocked, w2.sf_blocked, M, N, K,
                           acc=np.float64)
    np.testing.assert_allclose(d.astype(np.float64), d64, rtol=1e-2, atol=1e-2)


def test_grouped_sizes_seed0(pkg):
    assert pkg.inputs.grouped_m_sizes(8, seed=0) == [832, 1024, 384, 64, 256, 768, 256, 512]
