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


def _allgather(pkg, x, rows, outs, flags, world, rank, epoch, m_off=0):
    import ctypes
    VP = ctypes.c_void_p
    peer_out = (VP * world)(*[o.data_ptr() for o in outs])
    peer_flag = (VP * world)(*[f.data_ptr() for f in flags])
    sa, sb, ssa, ssb = x.a.stride(), x.b.stride(), x.sfa.stride(), x.sfb.stride()
    return pkg._lib.lib().nvfp4_gemv_allgather(
        x.a.data_ptr(), x.b.data_ptr(), x.sfa.data_ptr(), x.sfb.data_ptr(), rows, x.K, x.L,
        sa[0], sa[2], sb[2], ssa[0], ssa[2], ssb[2], peer_out, 1, x.M, m_off, peer_flag, world, rank, epoch,
        torch.cuda.current_stream().cuda_stream)


def test_fused_gather_peer_wait_expires_and_recovers(pkg, oracle, cuda):
    """One GPU plays rank 0 of a 2-rank fused all-gather whose rank 1 never
    delivers: both 'peer' buffers are local, and nothing writes rank 1's epoch.
    With a 1 ms budget the completion wait must give up, set the peer-timeout
    bit (16) and leave rank 0's rows in both buffers.  The same flag buffers then
    complete a second call once rank 1's epoch is present, and the default
    budget is restored."""
    M, K, L = 512, 2048, 1
    x = pkg.inputs.gemv_inputs(M, K, L, seed=5, device=cuda)
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    want = x.c[:, 0, 0].clone()
    half = M // 2
    xr = pkg.inputs.GemvInputs(x.a[:half], x.b, x.sfa[:half], x.sfb, None, M, K, L)
    outs = [torch.full((M,), float("nan"), dtype=torch.float16, device=cuda) for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device=cuda) for _ in range(2)]
    pkg._lib.device_errors(clear=True)
    pkg._lib.check(pkg._lib.lib().nvfp4_set_peer_wait_ns(1_000_000))
    try:
        pkg._lib.check(_allgather(pkg, xr, half, outs, flags, 2, 0, epoch=1))
        torch.cuda.synchronize()
        assert pkg._lib.device_errors(clear=True) & (1 << 4)
        for o in outs:   # rank 0's rows reached both buffers; rank 1's never came
            assert torch.equal(o[:half], want[:half])
            assert torch.isnan(o[half:]).all()
        f0 = flags[0].cpu()
        assert f0[0] == 1 and f0[1] == 0 and flags[1].cpu()[0] == 1   # epoch published to both
        assert f0[16] == 0                                             # CTA counter reset for the next call
        stamps = f0[32:38].numpy().view(np.uint32).astype(np.uint64)
        t_start, t_pub, t_end = (int(stamps[2 * i]) | (int(stamps[2 * i + 1]) << 32) for i in range(3))
        assert t_start <= t_pub <= t_end and t_end - t_pub >= 1_000_000
        # rank 1 "arrives" for call 2: the same buffers complete without error
        flags[0][1] = 2
        pkg._lib.check(_allgather(pkg, xr, half, outs, flags, 2, 0, epoch=2))
        torch.cuda.synchronize()
        assert pkg._lib.device_errors(clear=True) == 0
    finally:
        pkg._lib.check(pkg._lib.lib().nvfp4_set_peer_wait_ns(0))
    with pytest.raises(RuntimeError, match="budget"):
        pkg._lib.check(pkg._lib.lib().nvfp4_set_peer_wait_ns(10))
    # the context still computes
    x.c.zero_()
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    assert torch.equal(x.c[:, 0, 0], want)
