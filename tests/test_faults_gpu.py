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


def _allgather(pkg, x, rows, out, stages, world, rank, epoch, m_off=0):
    import ctypes
    VP = ctypes.c_void_p
    peer_stage = (VP * world)(*[t.data_ptr() for t in stages])
    sa, sb, ssa, ssb = x.a.stride(), x.b.stride(), x.sfa.stride(), x.sfb.stride()
    return pkg._lib.lib().nvfp4_gemv_allgather(
        x.a.data_ptr(), x.b.data_ptr(), x.sfa.data_ptr(), x.sfb.data_ptr(), rows, x.K, x.L,
        sa[0], sa[2], sb[2], ssa[0], ssa[2], ssb[2], out.data_ptr(), 1, x.M, m_off, x.M, peer_stage, world, rank,
        epoch, torch.cuda.current_stream().cuda_stream)


def _lines(stage, M):
    """The 64-bit lines of a staging buffer for an even M: (epoch per line,
    fp16 bits per element; two elements per line, low half first)."""
    v = stage[64: 64 + M].cpu().numpy().view(np.uint64)
    ep = (v >> np.uint64(32)).astype(np.uint32)
    bits = np.stack([(v & np.uint64(0xFFFF)), (v >> np.uint64(16)) & np.uint64(0xFFFF)], axis=1)
    return ep, bits.astype(np.uint16).reshape(-1)


def test_fused_gather_peer_wait_expires_and_recovers(pkg, oracle, cuda):
    """One GPU plays rank 0 of a 2-rank fused all-gather whose rank 1 never
    delivers: both staging buffers are local, and nothing writes rank 1's rows.
    With a 1 ms budget the waits for those rows must give up, set the
    peer-timeout bit (16), and leave rank 0's rows in the output and in both
    staging buffers.  The same buffers then complete a second call once rank
    1's lines for it are present, and the default budget is restored."""
    M, K, L = 512, 2048, 1
    x = pkg.inputs.gemv_inputs(M, K, L, seed=5, device=cuda)
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    want = x.c[:, 0, 0].clone()
    half = M // 2
    xr = pkg.inputs.GemvInputs(x.a[:half], x.b, x.sfa[:half], x.sfb, None, M, K, L)
    out = torch.full((M,), float("nan"), dtype=torch.float16, device=cuda)
    stages = [torch.zeros(64 + 2 * M, dtype=torch.int32, device=cuda) for _ in range(2)]
    pkg._lib.device_errors(clear=True)
    pkg._lib.check(pkg._lib.lib().nvfp4_set_peer_wait_ns(1_000_000))
    try:
        pkg._lib.check(_allgather(pkg, xr, half, out, stages, 2, 0, epoch=1))
        torch.cuda.synchronize()
        assert pkg._lib.device_errors(clear=True) & (1 << 4)
        assert torch.equal(out[:half], want[:half])          # rank 0's rows arrived
        assert torch.isnan(out[half:]).all()                 # rank 1's never came
        want_bits = want.cpu().numpy().view(np.uint16)
        for st in stages:                                    # rank 0 sent its lines to both ranks
            ep, bits = _lines(st, M)
            assert (ep[: half // 2] == 1).all() and (ep[half // 2:] == 0).all()
            assert np.array_equal(bits[:half], want_bits[:half])
        ctl = stages[0].cpu()
        assert ctl[16] == 0                                  # CTA count reset for the next call
        w = ctl[32:38].numpy().view(np.uint32).astype(np.uint64)
        t_start, t_sent, t_end = (int(w[2 * i]) | (int(w[2 * i + 1]) << 32) for i in range(3))
        assert t_start <= t_sent <= t_end and t_end - t_start >= 1_000_000
        # rank 1 "delivers" its rows of call 2: the same buffers complete it without error
        pairs = want_bits[half:].astype(np.uint64).reshape(-1, 2)
        lines = (np.uint64(2) << np.uint64(32)) | pairs[:, 0] | (pairs[:, 1] << np.uint64(16))
        stages[0][64 + half: 64 + M] = torch.from_numpy(lines.view(np.int32)).to(cuda)
        out.fill_(float("nan"))
        pkg._lib.check(_allgather(pkg, xr, half, out, stages, 2, 0, epoch=2))
        torch.cuda.synchronize()
        assert pkg._lib.device_errors(clear=True) == 0
        assert torch.equal(out, want)
    finally:
        pkg._lib.check(pkg._lib.lib().nvfp4_set_peer_wait_ns(0))
    with pytest.raises(RuntimeError, match="budget"):
        pkg._lib.check(pkg._lib.lib().nvfp4_set_peer_wait_ns(10))
    # the context still computes
    x.c.zero_()
    pkg.custom_kernel(*x.as_tuple())
    torch.cuda.synchronize()
    assert torch.equal(x.c[:, 0, 0], want)


def test_fused_gather_world1_matches_plain_kernel(pkg, cuda):
    """A 1-rank fused launch (staging buffer local) returns exactly the plain
    kernel's output, call after call, and in device-epoch mode too."""
    for M, K, L in ((16384, 16384, 1), (1000, 2048, 3), (999, 2048, 2)):   # two / one result(s) per line
        x = pkg.inputs.gemv_inputs(M, K, L, seed=2, device=cuda)
        pkg.custom_kernel(*x.as_tuple())
        torch.cuda.synchronize()
        want = x.c.permute(2, 1, 0).contiguous().view(-1)
        stage = torch.zeros(64 + 2 * M * L, dtype=torch.int32, device=cuda)
        out = torch.empty(M * L, dtype=torch.float16, device=cuda)
        import ctypes
        peer = (ctypes.c_void_p * 1)(stage.data_ptr())
        sa, sb, ssa, ssb = x.a.stride(), x.b.stride(), x.sfa.stride(), x.sfb.stride()
        for epoch in (1, 2, 3, 0, 0):
            out.fill_(float("nan"))
            pkg._lib.check(pkg._lib.lib().nvfp4_gemv_allgather(
                x.a.data_ptr(), x.b.data_ptr(), x.sfa.data_ptr(), x.sfb.data_ptr(), M, K, L,
                sa[0], sa[2], sb[2], ssa[0], ssa[2], ssb[2], out.data_ptr(), 1, M, 0, M, peer, 1, 0, epoch,
                torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
            assert torch.equal(out, want), (M, epoch)
        assert pkg._lib.device_errors() == 0
