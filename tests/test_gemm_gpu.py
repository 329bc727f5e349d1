"""GPU parity of the tcgen05 NVFP4 GEMMs (dual SiLU-gate, grouped) against the
CPU oracle (fp32 dequantise-then-matmul), rtol = atol = 1e-2 on fp16 outputs.
No reference kernel exists for these two: parity is pinned by the oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2


def _ops(pkg, rows_list, K, seed):
    g = torch.Generator().manual_seed(seed)
    return [pkg.inputs.operand(r, K, g) for r in rows_list]


def _close(got, ref):
    np.testing.assert_allclose(got.astype(np.float32), ref.astype(np.float32), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("M,N,K", [
    (128, 128, 256),        # one tile, one K step
    (256, 14336, 4096),     # config 3 at full size
    (200, 384, 320),        # M tail, K with a partial last step
    (64, 1000, 1024),       # N tail, small M
    (1, 128, 64),           # one row, one MMA
])
def test_dual_gemm(pkg, oracle, cuda, M, N, K):
    x, w1, w2 = _ops(pkg, [M, N, N], K, seed=M * 7 + N + K)
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
    d = lambda t: t.to(cuda)
    pkg.dual_gemm(d(x.codes), d(w1.codes), d(w2.codes), d(x.sf_blocked), d(w1.sf_blocked), d(w2.sf_blocked), c)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    ref = oracle.dual_gemm(x.codes, w1.codes, w2.codes, x.sf_blocked, w1.sf_blocked, w2.sf_blocked, M, N, K)
    _close(c.cpu().numpy(), ref)


def _grouped(pkg, oracle, cuda, Ms, N, K, seed, ldc_pad=0):
    ops = _ops(pkg, [m for m in Ms for _ in (0,)] + [N] * len(Ms), K, seed)
    As, Bs = ops[: len(Ms)], ops[len(Ms):]
    cs_full = [torch.full((m, N + ldc_pad), float("nan"), dtype=torch.float16, device=cuda) for m in Ms]
    cs = [c[:, :N] for c in cs_full]
    pkg.grouped_gemm([a.codes.to(cuda) for a in As], [b.codes.to(cuda) for b in Bs],
                     [a.sf_blocked.to(cuda) for a in As], [b.sf_blocked.to(cuda) for b in Bs], cs)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    for m, a, b, c in zip(Ms, As, Bs, cs):
        if m == 0:
            continue
        _close(c.cpu().numpy(), oracle.gemm(a.codes, b.codes, a.sf_blocked, b.sf_blocked, m, N, K).astype(np.float16))
    return cs_full


def test_grouped_gemm_config4(pkg, oracle, cuda):
    Ms = pkg.inputs.grouped_m_sizes(8, seed=0)
    _grouped(pkg, oracle, cuda, Ms, 4096, 7168, seed=0)


@pytest.mark.parametrize("Ms,N,K", [([128], 256, 256), ([100, 1, 300, 129], 384, 512), ([64, 64], 200, 128)])
def test_grouped_gemm_ragged(pkg, oracle, cuda, Ms, N, K):
    _grouped(pkg, oracle, cuda, Ms, N, K, seed=sum(Ms))


def test_grouped_gemm_empty_group_and_unaligned_ldc(pkg, oracle, cuda):
    """A group with M = 0 is skipped; ldc = N + 3 forces element stores; the
    padding columns stay untouched."""
    cs = _grouped(pkg, oracle, cuda, [96, 0, 130], 256, 256, seed=5, ldc_pad=3)
    for c in cs:
        if c.shape[0]:
            assert torch.isnan(c[:, 256:]).all()


def test_grouped_gemm_many_groups(pkg, oracle, cuda):
    """More than one launch's worth of groups (24 per launch)."""
    _grouped(pkg, oracle, cuda, [64] * 40, 128, 128, seed=40)


def test_gemm_rejects_bad_inputs(pkg, cuda):
    x, w = _ops(pkg, [128, 128], 256, seed=1)
    c = torch.empty((128, 128), dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        pkg.grouped_gemm([x.codes.to(cuda)], [w.codes.to(cuda)], [x.sf_blocked[:100].to(cuda)],
                         [w.sf_blocked.to(cuda)], [c])
    with pytest.raises(RuntimeError, match="multiple of 64"):
        a = torch.zeros((128, 16), dtype=torch.uint8, device=cuda)   # K = 32
        s = torch.zeros(512, dtype=torch.uint8, device=cuda)
        pkg.grouped_gemm([a], [a], [s], [s], [c])


def test_plain_scales_are_converted(pkg, oracle, cuda):
    """Scales given as plain [rows, K/16] are converted to the blocked layout."""
    M, N, K = 128, 256, 512
    x, w = _ops(pkg, [M, N], K, seed=2)
    sa = pkg.layout.from_blocked(x.sf_blocked, M, K // 16)
    sb = pkg.layout.from_blocked(w.sf_blocked, N, K // 16)
    c = torch.empty((M, N), dtype=torch.float16, device=cuda)
    pkg.grouped_gemm([x.codes.to(cuda)], [w.codes.to(cuda)], [sa.to(cuda)], [sb.to(cuda)], [c])
    torch.cuda.synchronize()
    _close(c.cpu().numpy(), oracle.gemm(x.codes, w.codes, x.sf_blocked, w.sf_blocked, M, N, K).astype(np.float16))


def test_mma_peak_probe_runs(pkg, cuda):
    s = torch.cuda.current_stream().cuda_stream
    pkg._lib.check(pkg._lib.lib().nvfp4_mma_peak(64, s))
    pkg._lib.check(pkg._lib.lib().nvfp4_mma_peak_pattern(64, 1, s))
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    with pytest.raises(RuntimeError, match="pattern"):
        pkg._lib.check(pkg._lib.lib().nvfp4_mma_peak_pattern(64, 2, s))


@pytest.mark.parametrize("T,N,K", [(1, 4096, 4096), (8, 14336, 4096), (16, 1000, 512), (17, 640, 256), (64, 256, 1024),
                                   (3, 130, 64)])
def test_skinny_gemm(pkg, oracle, cuda, T, N, K):
    x, w = _ops(pkg, [T, N], K, seed=T * 31 + N)
    out = torch.full((T, N), float("nan"), dtype=torch.float16, device=cuda)
    pkg.skinny_gemm(x.codes.to(cuda), w.codes.to(cuda), x.sf_blocked.to(cuda), w.sf_blocked.to(cuda), out)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    ref = oracle.gemm(x.codes, w.codes, x.sf_blocked, w.sf_blocked, T, N, K).astype(np.float16)
    _close(out.cpu().numpy(), ref)


def test_skinny_gemm_rejects_too_many_rows(pkg, cuda):
    x, w = _ops(pkg, [65, 128], 64, seed=3)
    out = torch.empty((65, 128), dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        pkg.skinny_gemm(x.codes.to(cuda), w.codes.to(cuda), x.sf_blocked.to(cuda), w.sf_blocked.to(cuda), out)
