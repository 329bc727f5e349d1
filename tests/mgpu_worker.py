"""Worker for tests/test_multigpu_gpu.py, run under torch.distributed.run (one
rank per GPU, NCCL).  Rank-sharded GEMV through (1) local kernel + NCCL
all-gather and (2) the fused peer-store all-gather, against the single-GPU
kernel on the full problem.  Prints one line 'RANK r OK' or raises."""
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    for (M, K, L) in [(16384, 16384, 1), (1000, 2048, 3), (4096, 14336, 8)]:
        full = pkg.inputs.gemv_inputs(M, K, L, seed=0, device="cuda")
        pkg.custom_kernel(*full.as_tuple())
        ref = full.c.float()
        lo, hi = pkg.sharded.row_split(M, world, rank)
        sub = lambda t: t[lo:hi].permute(2, 0, 1).contiguous().permute(1, 2, 0)
        a, sfa = sub(full.a), sub(full.sfa)
        sh = pkg.sharded.ShardedGemv(M, K, L)
        sh(pkg.custom_kernel, a, full.b, sfa, full.sfb)
        torch.cuda.synchronize()
        nccl = sh.full().float()
        fused = pkg.sharded.FusedShardedGemv(M, K, L)
        for _ in range(3):                  # repeated calls exercise the running counter target
            out = fused(a, full.b, sfa, full.sfb)
        torch.cuda.synchronize()
        got = out.float()
        assert pkg._lib.device_errors() == 0, "device error word set"
        assert torch.equal(got, nccl), f"fused vs NCCL mismatch at M={M} K={K} L={L}"
        assert torch.allclose(got, ref, rtol=1e-2, atol=1e-2), f"sharded vs single-GPU mismatch {M} {K} {L}"
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
            assert torch.equal(gfused.out().float(), nccl), f"graph replay mismatch {M} {K} {L}"
        assert pkg._lib.device_errors() == 0, "device error word set after graph replays"
        dist.barrier()
    print(f"RANK {rank} OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
