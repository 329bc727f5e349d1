"""The allocation-free self-test entry point, nvfp4_selftest_wait_timeout_noalloc.

It is meant for callers that cannot allocate device memory (a serving process
whose allocator already owns the whole GPU, a host runtime without a device
allocation hook): it keeps its outcome words in a fixed array inside the
library instead of allocating them per call.

This file is collected last, so a run that stops at the first failure has run
every other test before it.  It passes alone in a fresh process and after the
rest of the suite.  Through the C ABI it runs the existing entry point
(nvfp4_selftest_wait_timeout) and the new one twice in a row, and checks that
they report the same outcome: the status code, every wait expiring, the same
device error bit, and a context that still computes afterwards.  The results
are integers, so the comparison is exact.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT = 4
BUDGET_NS = 1_000_000        # 1 ms per wait
ERR_BIT_SELFTEST = 1 << 3


def _existing(pkg):
    pkg._lib.device_errors(clear=True)
    rc = pkg._lib.lib().nvfp4_selftest_wait_timeout(BUDGET_NS, torch.cuda.current_stream().cuda_stream)
    return rc, pkg._lib.device_errors(clear=True)


def _no_alloc(pkg, waiters):
    expired = ctypes.c_int(-1)
    rc = pkg._lib.lib().nvfp4_selftest_wait_timeout_noalloc(
        BUDGET_NS, waiters, ctypes.byref(expired), torch.cuda.current_stream().cuda_stream)
    return rc, expired.value, pkg._lib.device_errors(clear=True)


def test_no_alloc_selftest_matches_existing(pkg, cuda):
    rc_ref, bits_ref = _existing(pkg)
    assert rc_ref == TIMEOUT and bits_ref & ERR_BIT_SELFTEST
    for waiters in (1, 1):                    # two calls in a row share the library's words
        rc, expired, bits = _no_alloc(pkg, waiters)
        assert (rc, bits) == (rc_ref, bits_ref)
        assert expired == waiters
    for waiters in (8, 64):                   # several waiting blocks, up to the array's size
        rc, expired, bits = _no_alloc(pkg, waiters)
        assert rc == TIMEOUT and expired == waiters and bits == bits_ref


def test_no_alloc_selftest_rejects_oversize(pkg, cuda):
    expired = ctypes.c_int(-1)
    rc = pkg._lib.lib().nvfp4_selftest_wait_timeout_noalloc(BUDGET_NS, 65, ctypes.byref(expired), None)
    assert rc == 1 and b"64" in pkg._lib.lib().nvfp4_last_error()
    assert expired.value == -1


def test_context_still_computes_after_no_alloc_selftest(pkg, oracle, cuda):
    x = pkg.inputs.gemv_inputs(64, 512, 1, seed=2, device=cuda)
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    ref = oracle.gemv(*(t.cpu() for t in (x.a, x.b, x.sfa, x.sfb)), 64, 512, 1)
    np.testing.assert_allclose(x.c.cpu().numpy().astype(np.float32), ref.astype(np.float32), rtol=1e-2, atol=1e-2)
    assert pkg._lib.device_errors() == 0
