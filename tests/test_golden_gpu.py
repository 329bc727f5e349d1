"""The CUDA GEMV on the reference kernel's own known-answer fixtures.

tests/golden/ holds outputs of the reference kernel (blackwell_nvfp4_gemv.cu,
built from its source; decode path :85-98) made by tests/golden/make_golden.py:

* kat_e2m1.npz: the full 16 x 16 product table of the e2m1 decode;
* kat_e4m3.npz: every one of the 256 e4m3 scale bytes, 0x7F / 0xFF being NaN;
* config0.npz: the seeded config-0 problem (M=256, K=1024, L=1).

Both known-answer results are exactly representable, so the library must
reproduce them bit for bit through custom_kernel (NaN exactly where the
reference has NaN).  For config 0 the reference rounds chunk sums in f16
(:126-131); the library must sit within 1 fp16 ulp of the exact result and
within the contract tolerance of the reference's output.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _run_fixture(pkg, cuda, name):
    d = np.load(os.path.join(GOLD, name))
    M, K, L = (int(v) for v in d["shape"])
    # [rows, cols, L] arrays -> L-outermost device tensors viewed as [rows, cols, L]
    dev = lambda t: torch.from_numpy(np.ascontiguousarray(t.transpose(2, 0, 1))).to(cuda).permute(1, 2, 0)
    c = torch.full((L, 1, M), float("nan"), dtype=torch.float16, device=cuda).permute(2, 1, 0)
    pkg.custom_kernel(dev(d["a"]), dev(d["b"]), dev(d["sfa"]), dev(d["sfb"]), c)
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    return d, c.cpu().numpy(), (M, K, L)


def test_kat_e2m1_bit_exact(pkg, cuda):
    d, got, _ = _run_fixture(pkg, cuda, "kat_e2m1.npz")
    np.testing.assert_array_equal(got.view(np.uint16), d["c"].view(np.uint16))


def test_kat_e4m3_all_bytes_bit_exact(pkg, cuda):
    d, got, _ = _run_fixture(pkg, cuda, "kat_e4m3.npz")
    ref = d["c"]
    nan = np.isnan(ref)
    assert nan[0x7F, 0, 0] and nan[0xFF, 0, 0] and nan.sum() == 2
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint16), ref[~nan].view(np.uint16))


def test_config0_against_reference_fixture(pkg, oracle, cuda):
    d, got, (M, K, L) = _run_fixture(pkg, cuda, "config0.npz")
    got = got.astype(np.float64)
    exact = oracle.gemv(d["a"], d["b"], d["sfa"], d["sfb"], M, K, L, acc=np.float64)
    ulp = np.abs(np.spacing(exact.astype(np.float16))).astype(np.float64)
    assert (np.abs(got - exact) <= ulp + 1e-9).all()
    ref = d["c"].astype(np.float64)
    # the reference's f16 chunk sums bound its error by the output scale
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()
    assert np.isclose(got, ref, rtol=1e-2, atol=1e-2).mean() >= 0.99
