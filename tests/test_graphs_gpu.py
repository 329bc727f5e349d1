"""Every operator can be captured into a CUDA graph and replayed: the library
launches on the caller's stream, encodes its tensor maps on the host at
capture time, and allocates nothing, so a replay recomputes the same results
bit for bit (row f3: graph capture of the hot path)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _replay_matches(fn, outs):
    """Runs fn eagerly, captures it, clears the outputs, replays twice and
    compares bit for bit with the eager results."""
    fn()
    torch.cuda.synchronize()
    want = [o.clone() for o in outs]
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()                                  # warm up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        fn()
    for _ in range(2):
        for o in outs:
            o.fill_(float("nan")) if o.is_floating_point() else o.fill_(0)
        g.replay()
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            assert torch.equal(o, w)


def test_graph_gemv(pkg, cuda):
    x = pkg.inputs.gemv_inputs(4096, 14336, 2, seed=3, device=cuda)
    _replay_matches(lambda: pkg.custom_kernel(*x.as_tuple()), [x.c])
    assert pkg._lib.device_errors() == 0


def test_graph_gemms_and_quantiser(pkg, cuda):
    g = torch.Generator().manual_seed(4)
    op = lambda r, k: pkg.inputs.operand(r, k, g, device=cuda)
    x, w1, w2 = op(256, 1024), op(512, 1024), op(512, 1024)
    c = torch.empty((256, 512), dtype=torch.float16, device=cuda)
    _replay_matches(lambda: pkg.dual_gemm(x.codes, w1.codes, w2.codes, x.sf_blocked, w1.sf_blocked,
                                          w2.sf_blocked, c), [c])
    Ms = [128, 64, 300]
    As, Bs = [op(m, 512) for m in Ms], [op(256, 512) for _ in Ms]
    cs = [torch.empty((m, 256), dtype=torch.float16, device=cuda) for m in Ms]
    _replay_matches(lambda: pkg.grouped_gemm([a.codes for a in As], [b.codes for b in Bs],
                                             [a.sf_blocked for a in As], [b.sf_blocked for b in Bs], cs), cs)
    t, w = op(16, 1024), op(1000, 1024)
    out = torch.empty((16, 1000), dtype=torch.float16, device=cuda)
    _replay_matches(lambda: pkg.skinny_gemm(t.codes, w.codes, t.sf_blocked, w.sf_blocked, out), [out])
    xf = torch.randn((300, 2048), generator=g).to(torch.float16).to(cuda)
    codes = torch.empty((300, 1024), dtype=torch.uint8, device=cuda)
    sf = torch.empty(pkg.layout.blocked_numel(300, 128), dtype=torch.uint8, device=cuda)
    _replay_matches(lambda: pkg.quantize(xf, codes, sf), [codes, sf])
    assert pkg._lib.device_errors() == 0
