"""The NVFP4 quantiser: CPU checks of the oracle's rounding rules, and GPU
bit-exactness of the kernel against the oracle (codes and blocked scales are
bytes: exact equality is the bar), plus quantise -> dual GEMM end to end.
No reference code exists for quantisation (the reference's inputs arrive
already quantised), so parity is pinned by the oracle's restatement."""
import numpy as np
import pytest
import torch


def test_oracle_e2m1_rounding(oracle):
    v = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.0, -0.3, -5.0, 0.26, 1e9])
    assert oracle.e2m1_rne_satfinite(v).tolist() == [0, 2, 2, 4, 4, 6, 6, 7, 8, 9, 14, 1, 7]
    grid = oracle.E2M1_LUT
    for c in range(16):   # every code value round-trips
        assert oracle.e2m1_rne_satfinite(np.array([grid[c]]))[0] == (0 if c == 0 else (8 if c == 8 else c))


def test_oracle_e4m3_rounding(oracle):
    vals = oracle.E4M3_LUT[:0x7F].astype(np.float64)
    assert (oracle.e4m3_rne_satfinite(vals) == np.arange(0x7F)).all()
    assert oracle.e4m3_rne_satfinite(np.array([1000.0, 449.0]))[0] == 0x7E          # saturates at 448
    assert oracle.e4m3_rne_satfinite(np.array([2.0 ** -10]))[0] == 0                 # tie below 2^-9 -> 0
    assert oracle.e4m3_rne_satfinite(np.array([1.0625]))[0] == 0x38                  # 1 + 1/16: tie -> even (1.0)


def test_oracle_e4m3_matches_torch_cast(oracle):
    """Independent pin of the oracle's e4m3 rounding: for 200k random finite
    values inside the e4m3 range, round-to-nearest-even must give the same byte
    as torch's own float8_e4m3fn cast (which rounds to nearest even; the range
    is kept inside +-448 because the cast does not saturate)."""
    rng = np.random.default_rng(1)
    mag = np.exp2(rng.uniform(-12, np.log2(448.0), 200_000))
    x = (mag * rng.choice([-1.0, 1.0], mag.size)).astype(np.float32)
    x[:6] = [0.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 448.0, 1.0625]   # ties and edges
    ours = oracle.e4m3_rne_satfinite(np.abs(x).astype(np.float64)).astype(np.uint8)
    theirs = torch.from_numpy(np.abs(x)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, theirs)


def test_oracle_e2m1_matches_brute_force(oracle):
    """The e2m1 rounding cross-checked by brute force: nearest of the eight
    magnitudes by direct distance, ties to the even code, saturation at 6."""
    rng = np.random.default_rng(2)
    v = rng.uniform(-8, 8, 100_000)
    grid = np.array([0, .5, 1, 1.5, 2, 3, 4, 6])
    v[:16] = np.concatenate([(grid[1:] + grid[:-1]) / 2, [-0.25, 6.5, -7, 0, 5.0, 2.5, 0.75, 1.25, 1.75][:9]])
    a = np.minimum(np.abs(v), 6.0)
    d = np.abs(a[:, None] - grid[None, :])
    best = d.min(axis=1, keepdims=True)
    cand = np.where(d == best, np.arange(8)[None, :], 99)
    even = np.where(cand % 2 == 0, cand, 99).min(axis=1)
    mag = np.where(even < 99, even, cand.min(axis=1))
    want = (mag | np.where(np.signbit(v), 8, 0)).astype(np.uint8)
    np.testing.assert_array_equal(oracle.e2m1_rne_satfinite(v), want)


def test_oracle_quantize_roundtrip(pkg, oracle):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((64, 256)) * 3).astype(np.float16)
    codes, sf = oracle.quantize(x)
    deq = oracle.dequant_matrix(codes, sf, 64, 256)
    blocks = x.astype(np.float32).reshape(64, 16, 16)
    amax = np.abs(blocks).max(axis=2, keepdims=True)
    err = np.abs(deq.reshape(64, 16, 16) - blocks)
    assert (err <= amax * 0.25 + 1e-6).all()       # half an e2m1 step at the top of the block, plus scale rounding
    # values already on the grid of a power-of-two scale come back exactly
    grid = np.tile(np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -6, -4, -3, -2, -1.5, -1, -.5, 0], np.float32), (4, 4))
    c2, s2 = oracle.quantize(grid.astype(np.float16))
    np.testing.assert_array_equal(oracle.dequant_matrix(c2, s2, 4, 64), grid)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,scale", [(256, 4096, 1.0), (130, 80, 100.0), (7, 16, 1e-3), (300, 1024, 3e4)])
def test_quantize_bit_exact(pkg, oracle, cuda, M, K, scale):
    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn((M, K), generator=g) * scale).clamp(-65504, 65504).to(torch.float16)
    x[0, :16] = 0                         # all-zero block
    x[min(1, M - 1), :16] = -0.0          # negative zeros
    if K >= 32:
        x[min(2, M - 1), 16:32] = 6e-8    # fp16 subnormals: scale rounds to zero
    x[M - 1, -16:] = 65504                # largest fp16: the scale saturates at 448
    codes, sf = pkg.quantize(x.to(cuda))
    torch.cuda.synchronize()
    rc, rs = oracle.quantize(x.numpy())
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(sf.cpu().numpy(), rs)


@pytest.mark.gpu
def test_quantize_strided_input(pkg, oracle, cuda):
    g = torch.Generator().manual_seed(9)
    big = torch.randn((64, 600), generator=g).to(torch.float16)
    x = big[:, 8:520]                     # row stride 600 elements, base offset 16 bytes
    codes, sf = pkg.quantize(big.to(cuda)[:, 8:520])
    torch.cuda.synchronize()
    rc, rs = oracle.quantize(x.numpy())
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(sf.cpu().numpy(), rs)


@pytest.mark.gpu
def test_quantize_odd_alignment(pkg, oracle, cuda):
    """A row stride and base offset that are odd in elements: 2-byte aligned input rows."""
    g = torch.Generator().manual_seed(13)
    big = torch.randn((40, 1043), generator=g).to(torch.float16)
    x = big[:, 1:1025]                    # base offset 2 bytes, row stride 1043 elements
    codes, sf = pkg.quantize(big.to(cuda)[:, 1:1025])
    torch.cuda.synchronize()
    rc, rs = oracle.quantize(x.numpy())
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(sf.cpu().numpy(), rs)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(129, 16400), (3, 32784)])
def test_quantize_long_rows(pkg, oracle, cuda, M, K):
    """Rows longer than one CTA's 1024 blocks (the threads loop over the row)."""
    g = torch.Generator().manual_seed(M)
    x = torch.randn((M, K), generator=g).to(torch.float16)
    codes, sf = pkg.quantize(x.to(cuda))
    torch.cuda.synchronize()
    rc, rs = oracle.quantize(x.numpy())
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(sf.cpu().numpy(), rs)


@pytest.mark.gpu
def test_quantize_then_dual_gemm(pkg, oracle, cuda):
    M, N, K = 256, 1024, 1024
    g = torch.Generator().manual_seed(11)
    x = torch.randn((M, K), generator=g).to(torch.float16)
    xc, xs = pkg.quantize(x.to(cuda))
    w1, w2 = (pkg.inputs.operand(N, K, g) for _ in range(2))
    c = torch.empty((M, N), dtype=torch.float16, device=cuda)
    pkg.dual_gemm(xc, w1.codes.to(cuda), w2.codes.to(cuda), xs, w1.sf_blocked.to(cuda), w2.sf_blocked.to(cuda), c)
    torch.cuda.synchronize()
    ref = oracle.dual_gemm(xc.cpu(), w1.codes, w2.codes, xs.cpu(), w1.sf_blocked, w2.sf_blocked, M, N, K)
    np.testing.assert_allclose(c.cpu().numpy().astype(np.float32), ref.astype(np.float32), rtol=1e-2, atol=1e-2)
