"""GPU parity of the GEMV (through the C ABI) against the CPU oracle, the
reference kernel where it is built, and the edge cases of the reference's
input space.  Tolerance: rtol = atol = 1e-2 on fp16 outputs (north-star
contract); additionally the kernel must sit within 1 fp16 ulp of the exact
(float64) result, which its exact block sums guarantee."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2


def _run(pkg, x):
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    return x.c.cpu().numpy()


def _to_cpu(x):
    return [t.cpu() for t in (x.a, x.b, x.sfa, x.sfb)]


def _check(oracle, got, a, b, sfa, sfb, M, K, L, strict=True):
    ref = oracle.gemv(a, b, sfa, sfb, M, K, L)
    np.testing.assert_allclose(got.astype(np.float32), ref.astype(np.float32), rtol=RTOL, atol=ATOL)
    if strict:
        exact = oracle.gemv(a, b, sfa, sfb, M, K, L, acc=np.float64)
        fin = np.isfinite(exact) & (np.abs(exact) < 65000)
        e16 = exact[fin].astype(np.float16)
        ulp = np.abs(np.spacing(e16.astype(np.float16))).astype(np.float64)
        err = np.abs(got[fin].astype(np.float64) - exact[fin])
        assert (err <= ulp + 1e-6).all(), f"max err/ulp {np.max(err / ulp)}"


@pytest.mark.parametrize("M,K,L", [
    (256, 1024, 1),     # config 0
    (100, 1024, 1),     # M not a multiple of any tile
    (64, 3072, 2),      # K spans a full and a half stage
    (96, 1280, 3),      # last stage holds one 128-byte slice
    (1, 256, 1),        # tiny, bulk-copy path
    (1, 16, 1),         # tiny, plain-load path
    (33, 1040, 2),      # K % 256 != 0 -> plain-load path
    (7, 48, 5),
    (512, 16384, 1),
    (2048, 16384, 1),   # < 16 rows per SM, wide stages (the 8-rank share of config 1)
    (1000, 6144, 1),    # < 16 rows per SM, K/2 = 3072: 1 KB stages
    (4096, 16384, 1),   # < 32 rows per SM: two CTAs per SM (the 4-rank share of config 1)
    (3000, 8192, 1),    # same class, ragged last tile
])
def test_gemv_parity(pkg, oracle, cuda, M, K, L):
    x = pkg.inputs.gemv_inputs(M, K, L, seed=M + K + L, device=cuda)
    got = _run(pkg, x)
    _check(oracle, got, *_to_cpu(x), M, K, L)


@pytest.mark.parametrize("M,K,L", [(16384, 16384, 1), (4096, 14336, 8)])
def test_gemv_full_size_configs(pkg, oracle, cuda, M, K, L):
    """Configs 1 and 2 at full size against the (multi-threaded) torch oracle."""
    x = pkg.inputs.gemv_inputs(M, K, L, seed=0, device=cuda)
    got = _run(pkg, x).astype(np.float32)
    ref = oracle.gemv_torch(*_to_cpu(x), M, K, L).numpy().astype(np.float32)
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
    # run-to-run determinism, bit for bit
    x.c.zero_()
    again = _run(pkg, x).astype(np.float32)
    np.testing.assert_array_equal(got, again)


def test_gemv_strided_and_canary(pkg, oracle, cuda):
    """Padded row strides, a strided output, and guard bytes around c."""
    M, K, L = 200, 2048, 2
    g = torch.Generator().manual_seed(7)
    pad = 48
    a_big = torch.randint(0, 256, (L, M, K // 2 + pad), dtype=torch.uint8, generator=g)
    sfa_big = ((torch.randint(-3, 4, (L, M, K // 16 + pad), generator=g) + 7) << 3).to(torch.uint8)
    b = torch.randint(0, 256, (L, 3, K // 2), dtype=torch.uint8, generator=g)
    sfb = ((torch.randint(-3, 4, (L, 3, K // 16), generator=g) + 7) << 3).to(torch.uint8)
    a = a_big.to(cuda).permute(1, 2, 0)[:, : K // 2, :]
    sfa = sfa_big.to(cuda).permute(1, 2, 0)[:, : K // 16, :]
    bd, sfbd = b.to(cuda).permute(1, 2, 0), sfb.to(cuda).permute(1, 2, 0)
    guard = 64
    buf = torch.full((L, 1, 2 * M + 2 * guard), 12345.0, dtype=torch.float16, device=cuda)
    c = buf[:, :, guard: guard + 2 * M: 2].permute(2, 1, 0)   # c_sm = 2
    pkg.custom_kernel(a, bd, sfa, sfbd, c)
    torch.cuda.synchronize()
    hb = buf.cpu()
    assert (hb[:, :, :guard] == 12345.0).all() and (hb[:, :, guard + 2 * M:] == 12345.0).all()
    assert (hb[:, :, guard + 1: guard + 2 * M: 2] == 12345.0).all()
    _check(oracle, c.cpu().numpy(), a.cpu(), bd.cpu(), sfa.cpu(), sfbd.cpu(), M, K, L)


def test_gemv_unaligned_pointer_uses_plain_path(pkg, oracle, cuda):
    M, K, L = 64, 512, 1
    x = pkg.inputs.gemv_inputs(M, K + 16, L, seed=3, device=cuda)
    a = x.a[:, 8:, :]          # base pointer offset by 8 bytes
    sfa = x.sfa[:, 1:, :]
    b = x.b[:, 8:, :]
    sfb = x.sfb[:, 1:, :]
    pkg.custom_kernel(a, b, sfa, sfb, x.c)
    torch.cuda.synchronize()
    _check(oracle, x.c.cpu().numpy(), a.cpu(), b.cpu(), sfa.cpu(), sfb.cpu(), M, K, L)


def test_gemv_extreme_scales(pkg, oracle, cuda):
    """e4m3 448 on both sides (a product of 200704, which overflows the
    reference's f16 scale product), subnormal scales and a NaN scale."""
    M, K, L = 64, 512, 1
    x = pkg.inputs.gemv_inputs(M, K, L, seed=11, device=cuda)
    sfa = x.sfa.cpu().clone()
    sfb = x.sfb.cpu().clone()
    a = x.a.cpu().clone()
    sfa[0:8] = 0x7E
    sfb[:, 0:4] = 0x7E
    a[0:8, :, :] = 0x11          # codes 0.5 keep those rows finite
    sfa[8:16] = 0x01             # smallest subnormal, 2^-9
    sfa[16, 3, 0] = 0x7F         # NaN
    for t, src in ((x.sfa, sfa), (x.sfb, sfb), (x.a, a)):
        t.copy_(src.to(cuda))
    got = _run(pkg, x)
    ref = oracle.gemv(a, x.b.cpu(), sfa, sfb, M, K, L)
    assert np.isnan(got[16]).all() and np.isnan(ref[16]).all()
    keep = np.ones(M, dtype=bool)
    keep[16] = False
    np.testing.assert_allclose(got[keep].astype(np.float32), ref[keep].astype(np.float32), rtol=RTOL, atol=ATOL)


def test_gemv_rejects_bad_inputs(pkg, cuda):
    x = pkg.inputs.gemv_inputs(32, 256, 1, device=cuda)
    with pytest.raises(ValueError):
        pkg.custom_kernel(x.a, x.b, x.sfa[:, :8], x.sfb, x.c)
    with pytest.raises(TypeError):
        pkg.custom_kernel(x.a, x.b, x.sfa, x.sfb, x.c.float())
    with pytest.raises(ValueError):
        pkg.custom_kernel(x.a.cpu(), x.b, x.sfa, x.sfb, x.c)


def test_gemv_tuple_form_and_fp4_dtypes(pkg, oracle, cuda):
    x = pkg.inputs.gemv_inputs(128, 512, 2, seed=9, device=cuda)
    if hasattr(torch, "float4_e2m1fn_x2"):
        data = (x.a.view(torch.float4_e2m1fn_x2), x.b.view(torch.float4_e2m1fn_x2),
                x.sfa.view(torch.float8_e4m3fn), x.sfb.view(torch.float8_e4m3fn), x.c)
    else:
        data = x.as_tuple()
    out = pkg.custom_kernel(data)
    torch.cuda.synchronize()
    assert out is x.c
    _check(oracle, out.cpu().numpy(), *_to_cpu(x), 128, 512, 2)


def test_gemv_on_side_stream(pkg, oracle, cuda):
    x = pkg.inputs.gemv_inputs(300, 2048, 1, seed=4, device=cuda)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        pkg.custom_kernel(*x.as_tuple())
    s.synchronize()
    _check(oracle, x.c.cpu().numpy(), *_to_cpu(x), 300, 2048, 1)


def test_gemv_forward_matches_custom_kernel(pkg, oracle, cuda):
    """The reference's binding signature: the full problem equals custom_kernel
    bit for bit; a sub-problem (first M rows, first L batches) computes exactly
    those outputs and leaves the rest of c untouched."""
    M, K, L = 256, 1024, 2
    x = pkg.inputs.gemv_inputs(M, K, L, seed=7, device=cuda)
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    want = x.c.clone()
    c = torch.full_like(x.c, float("nan"))
    assert pkg.nvfp4_gemv_forward(x.a, x.b, x.sfa, x.sfb, c, M, K, L) is None
    torch.cuda.synchronize()
    assert torch.equal(c, want)
    c.fill_(float("nan"))
    pkg.nvfp4_gemv_forward(x.a, x.b, x.sfa, x.sfb, c, 200, K, 1)
    torch.cuda.synchronize()
    assert torch.equal(c[:200, :, :1], want[:200, :, :1])
    assert torch.isnan(c[200:]).all() and torch.isnan(c[:, :, 1:]).all()
    assert pkg._lib.device_errors() == 0


@pytest.mark.parametrize("M,K,L", [(16384, 16384, 1), (4096, 14336, 8), (1000, 2048, 3)])
def test_row_shares_are_bit_identical_to_single_gpu(pkg, cuda, M, K, L):
    """What a rank of an N-way row-sharded GEMV computes (its rows alone, with
    the launch shape chosen for that share) equals the single-GPU rows bit for
    bit, for N = 2, 4, 8: the stage width, which alone fixes the summation
    order, depends on K only."""
    x = pkg.inputs.gemv_inputs(M, K, L, seed=1, device=cuda)
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    full = x.c.clone()
    for world in (2, 4, 8):
        for rank in range(world):
            lo, hi = pkg.sharded.row_split(M, world, rank)
            sub = lambda t: t[lo:hi].permute(2, 0, 1).contiguous().permute(1, 2, 0)
            c = torch.empty((L, 1, hi - lo), dtype=torch.float16, device=cuda).permute(2, 1, 0)
            pkg.custom_kernel(sub(x.a), x.b, sub(x.sfa), x.sfb, c)
            torch.cuda.synchronize()
            assert torch.equal(c.view(torch.int16), full[lo:hi].view(torch.int16)), (world, rank)
