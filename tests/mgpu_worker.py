"""Worker for tests/test_multigpu_gpu.py, run under torch.distributed.run (one
rank per GPU, NCCL).

* Row-sharded GEMV through (1) the local kernel + NCCL all-gather and (2) the
  fused peer-store all-gather, eager and replayed from a CUDA graph: both must
  equal the single-GPU kernel's output on the full problem bit for bit (a
  row's bits depend only on K, never on the rank's share).
* Group-sharded grouped GEMM (config 4's groups, LPT-assigned, one padded NCCL
  all-gather): every group's output equals the single-GPU grouped GEMM's bit
  for bit (a tile's arithmetic does not depend on which launch computes it).

Prints one line 'RANK r OK' or raises."""
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def check_gemv(pkg, rank, world):
    for (M, K, L) in [(16384, 16384, 1), (1000, 2048, 3), (4096, 14336, 8)]:
        full = pkg.inputs.gemv_inputs(M, K, L, seed=0, device="cuda")
        pkg.custom_kernel(*full.as_tuple())
        ref = full.c.clone()
        lo, hi = pkg.sharded.row_split(M, world, rank)
        sub = lambda t: t[lo:hi].permute(2, 0, 1).contiguous().permute(1, 2, 0)
        a, sfa = sub(full.a), sub(full.sfa)
        sh = pkg.sharded.ShardedGemv(M, K, L)
        sh(pkg.custom_kernel, a, full.b, sfa, full.sfb)
        torch.cuda.synchronize()
        assert torch.equal(sh.full(), ref), f"NCCL-gathered vs single-GPU mismatch at M={M} K={K} L={L}"
        fused = pkg.sharded.FusedShardedGemv(M, K, L)
        # the fused gather splits rows at even boundaries (two results per line)
        fsub = lambda t: t[fused.lo:fused.hi].permute(2, 0, 1).contiguous().permute(1, 2, 0)
        a, sfa = fsub(full.a), fsub(full.sfa)
        for _ in range(3):                  # repeated calls reuse the staging buffers
            out = fused(a, full.b, sfa, full.sfb)
        torch.cuda.synchronize()
        assert pkg._lib.device_errors() == 0, "device error word set"
        assert torch.equal(out, ref), f"fused vs single-GPU mismatch at M={M} K={K} L={L}"
        # device-epoch mode, captured once in a CUDA graph and replayed
        gfused = pkg.sharded.FusedShardedGemv(M, K, L, device_epoch=True)
        gfused(a, full.b, sfa, full.sfb)                   # eager call (also sets up the launch)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph):
                gfused(a, full.b, sfa, full.sfb)
        torch.cuda.synchronize()
        for _ in range(3):
            gfused.out_flat.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(gfused.out(), ref), f"graph replay mismatch {M} {K} {L}"
        assert pkg._lib.device_errors() == 0, "device error word set after graph replays"
        dist.barrier()


def check_grouped(pkg, rank, world):
    N, K = 4096, 7168
    Ms = pkg.inputs.grouped_m_sizes(8, seed=0)
    g = torch.Generator().manual_seed(0)
    As = [pkg.inputs.operand(m, K, g, device="cuda") for m in Ms]
    Bs = [pkg.inputs.operand(N, K, g, device="cuda") for _ in Ms]
    ref = [torch.empty((m, N), dtype=torch.float16, device="cuda") for m in Ms]
    pkg.grouped_gemm([a.codes for a in As], [b.codes for b in Bs], [a.sf_blocked for a in As],
                     [b.sf_blocked for b in Bs], ref)
    sh = pkg.sharded.ShardedGroupedGemm(Ms, N, K)
    mine = sh.mine
    for _ in range(2):
        sh(pkg.grouped_gemm, [As[i].codes for i in mine], [Bs[i].codes for i in mine],
           [As[i].sf_blocked for i in mine], [Bs[i].sf_blocked for i in mine])
    torch.cuda.synchronize()
    assert pkg._lib.device_errors() == 0
    for i, (o, r) in enumerate(zip(sh.outputs(), ref)):
        assert torch.equal(o, r), f"grouped group {i} mismatch on rank {rank}"
    dist.barrier()


def main():
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    check_gemv(pkg, rank, world)
    check_grouped(pkg, rank, world)
    print(f"RANK {rank} OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
