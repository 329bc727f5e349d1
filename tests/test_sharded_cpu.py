"""Host-side sharding logic on CPU: row splits, LPT group assignment, and the
all-gather plumbing with world_size-2 gloo ranks (a fake kernel stands in for
the GPU one)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_row_split_covers_and_balances(pkg):
    for M in (1, 7, 256, 16384, 16385):
        for world in (1, 2, 3, 4, 8):
            parts = [pkg.sharded.row_split(M, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == M
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1
            assert pkg.sharded.padded_rows(M, world) == max(sizes)


def test_lpt_assignment(pkg):
    Ms = pkg.inputs.grouped_m_sizes(8, seed=0)     # [832, 1024, 384, 64, 256, 768, 256, 512]
    owner = pkg.sharded.lpt_assign(Ms, 2)
    loads = [sum(m for m, o in zip(Ms, owner) if o == r) for r in range(2)]
    assert sum(loads) == 4096 and max(loads) - min(loads) <= max(Ms)   # LPT keeps the gap below one group
    assert max(loads) <= 4 / 3 * 2048
    owner8 = pkg.sharded.lpt_assign(Ms, 8)
    assert sorted(owner8) == list(range(8))         # one group per rank
    assert pkg.sharded.lpt_assign([5, 5, 5], 2) == [0, 1, 0]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # row-sharded GEMV: a fake kernel writes row index + 1000*l
        M, K, L = 37, 64, 3
        sh = pkg.sharded.ShardedGemv(M, K, L, device=torch.device("cpu"))

        def fake_gemv(a, b, sa, sb, c):
            for i in range(sh.hi - sh.lo):
                for l in range(L):
                    c[i, 0, l] = float(sh.lo + i + 1000 * l)
        sh(fake_gemv, None, None, None, None)
        full = sh.full()
        expect = torch.tensor([[[m + 1000 * l for l in range(L)]] for m in range(M)], dtype=torch.float16)
        ok1 = torch.equal(full, expect)
        # group-sharded grouped GEMM: fake kernel fills group g with g + 1
        Ms, N = [5, 3, 0, 7], 4
        gs = pkg.sharded.ShardedGroupedGemm(Ms, N, 64, device=torch.device("cpu"))

        def fake_grouped(al, bl, sal, sbl, cl):
            for g, c in zip(gs.mine, cl):
                c.fill_(g + 1)
        gs(fake_grouped, [None] * len(gs.mine), None, None, None)
        outs = gs.outputs()
        ok2 = all(o.shape == (m, N) and bool((o == g + 1).all()) for g, (o, m) in enumerate(zip(outs, Ms)))
        q.put((rank, ok1, ok2))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_gloo_world2_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    assert sorted(res) == [(0, True, True), (1, True, True)]


def _failing_worker(rank, world, port, q):
    """Rank 1 leaves before the output all-gather (between steps, nothing in
    flight); rank 0 must see its gather fail within the process group's
    timeout instead of waiting forever."""
    import sys
    import time
    from datetime import timedelta
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    Ms, N = [5, 3, 7], 4
    gs = pkg.sharded.ShardedGroupedGemm(Ms, N, 64, device=torch.device("cpu"))
    fake = lambda al, bl, sal, sbl, cl: [c.fill_(1.0) for c in cl]
    gs(fake, [None] * len(gs.mine), None, None, None)      # one healthy step on both ranks
    if rank == 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()                                      # flush the message before leaving
        os._exit(0)                                          # leaves without joining step 2
    t0 = time.monotonic()
    try:
        gs(fake, [None] * len(gs.mine), None, None, None)
        q.put((rank, "completed", time.monotonic() - t0))
    except Exception as e:  # gloo reports the lost peer or the timeout
        q.put((rank, "raised " + type(e).__name__, time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.timeout(120)
def test_gloo_rank_failure_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res[1][1] == "left"
    assert res[0][1].startswith("raised"), res
    assert res[0][2] < 30.0, res    # well inside the test's own limit: the 5 s group timeout or an earlier reset
