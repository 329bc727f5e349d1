"""Bounded waits: a wait that nothing satisfies must expire, report through the
status code and the device error word, and leave the context usable.  No GPU
fault, trap or hang is caused: the kernel simply gives up after ~1 ms."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_timeout_reports_and_recovers(pkg, oracle, cuda):
    pkg._lib.device_errors(clear=True)
    rc = pkg._lib.lib().nvfp4_selftest_wait_timeout(1_000_000, None)
    assert rc == 4, pkg._lib.lib().nvfp4_last_error()
    assert pkg._lib.device_errors(clear=True) & (1 << 3)
    assert pkg._lib.device_errors(clear=True) == 0
    # the context still works
    x = pkg.inputs.gemv_inputs(64, 512, 1, seed=2, device=cuda)
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    ref = oracle.gemv(*(t.cpu() for t in (x.a, x.b, x.sfa, x.sfb)), 64, 512, 1)
    np.testing.assert_allclose(x.c.cpu().numpy().astype(np.float32), ref.astype(np.float32), rtol=1e-2, atol=1e-2)
