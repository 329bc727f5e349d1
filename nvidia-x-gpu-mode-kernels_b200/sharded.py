"""Multi-GPU sharding: GEMV by output rows, grouped GEMM by group.

One process per GPU (``torch.distributed``, NCCL over NVLink / NVSwitch).  The
reference has no distributed code; these follow the north-star plan: each rank
computes its own slice of the output into a local buffer and one NCCL
all-gather assembles the full fp16 output on every rank.  No input moves
between GPUs: every rank holds (or streams) only its own rows / groups.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def row_split(M: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Contiguous row range [lo, hi) of rank `rank`; boundaries are multiples of
    `align` (except the end).  Ranks get equal shares up to one `align` unit."""
    units = (M + align - 1) // align
    lo = units * rank // world * align
    hi = min(M, units * (rank + 1) // world * align)
    return lo, hi


def padded_rows(M: int, world: int) -> int:
    """Rows per rank of the padded all-gather buffer."""
    return max(hi - lo for lo, hi in (row_split(M, world, r) for r in range(world)))


class ShardedGemv:
    """Row-sharded GEMV for L = 1 or more.

    Rank r owns rows [lo, hi) of A / SFA (a view of the full problem's rows, or
    its own copy of them); b / SFB are replicated.  ``__call__`` runs the local
    GEMV into a padded local buffer and all-gathers the padded slices into
    ``out`` ([world * rows_pad, 1, L] fp16, contiguous over rows for each l),
    whose first M rows (``full()``) are the complete result.
    """

    def __init__(self, M: int, K: int, L: int, group=None, device=None):
        self.M, self.K, self.L = M, K, L
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.lo, self.hi = row_split(M, self.world, self.rank)
        self.rows_pad = padded_rows(M, self.world)
        dev = device or torch.device("cuda", torch.cuda.current_device())
        # local and gathered outputs, L-major so every slice is contiguous
        self.local = torch.zeros((L, 1, self.rows_pad), dtype=torch.float16, device=dev)
        self.gathered = torch.empty((self.world, L, self.rows_pad), dtype=torch.float16, device=dev)

    def __call__(self, gemv, a_rows, b, sfa_rows, sfb) -> torch.Tensor:
        """`gemv` is the package's ``custom_kernel``; a_rows / sfa_rows hold this
        rank's rows only ([hi - lo, K/2, L] and [hi - lo, K/16, L])."""
        n = self.hi - self.lo
        c = self.local[:, :, :n].permute(2, 1, 0)
        if n > 0:
            gemv(a_rows, b, sfa_rows, sfb, c)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered.view(-1), self.local.view(-1), group=self.group)
        else:
            self.gathered[0].copy_(self.local[:, 0, :])
        return self.gathered

    def full(self) -> torch.Tensor:
        """[M, 1, L] view of the assembled output (copy-free when world == 1)."""
        parts = []
        for r in range(self.world):
            lo, hi = row_split(self.M, self.world, r)
            parts.append(self.gathered[r, :, : hi - lo])
        return torch.cat(parts, dim=1).transpose(0, 1).unsqueeze(1)


def lpt_assign(costs: list[float], world: int) -> list[int]:
    """Longest-processing-time-first: each group (largest cost first) goes to
    the rank with the least assigned cost.  Deterministic on ties (lowest
    rank, then group index)."""
    load = [0.0] * world
    owner = [0] * len(costs)
    for g in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = min(range(world), key=lambda k: (load[k], k))
        owner[g] = r
        load[r] += costs[g]
    return owner


class ShardedGroupedGemm:
    """Grouped GEMM sharded by group across ranks.

    Groups are bin-packed onto ranks by FLOPs (``lpt_assign``); each rank runs
    one grouped launch over its own groups, writing into a flat fp16 buffer
    laid out group after group; one all-gather of the buffers (padded to the
    largest rank's size) lets every rank unpack every group's output.
    """

    def __init__(self, Ms, N: int, K: int, group=None, device=None):
        self.Ms, self.N, self.K = list(Ms), N, K
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.owner = lpt_assign([m * N * K for m in self.Ms], self.world)
        self.mine = [g for g in range(len(self.Ms)) if self.owner[g] == self.rank]
        sizes = [sum(self.Ms[g] * N for g in range(len(self.Ms)) if self.owner[g] == r) for r in range(self.world)]
        self.pad = max(max(sizes), 1)
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.local = torch.zeros(self.pad, dtype=torch.float16, device=dev)
        self.gathered = torch.empty(self.world * self.pad, dtype=torch.float16, device=dev)
        self.local_views = []
        off = 0
        for g in self.mine:
            self.local_views.append(self.local[off: off + self.Ms[g] * N].view(self.Ms[g], N))
            off += self.Ms[g] * N

    def __call__(self, grouped_gemm, a_list, b_list, sfa_list, sfb_list):
        """Lists hold this rank's groups only, in ``self.mine`` order."""
        if self.mine:
            grouped_gemm(a_list, b_list, sfa_list, sfb_list, self.local_views)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.local, group=self.group)
        else:
            self.gathered.copy_(self.local)
        return self.gathered

    def outputs(self):
        """Every group's [M_g, N] output, viewed from the gathered buffer."""
        offs = [0] * self.world
        out = [None] * len(self.Ms)
        for g, m in enumerate(self.Ms):
            r = self.owner[g]
            base = r * self.pad + offs[r]
            out[g] = self.gathered[base: base + m * self.N].view(m, self.N)
            offs[r] += m * self.N
        return out


class FusedShardedGemv:
    """Row-sharded GEMV whose output all-gather is fused into the kernel.

    Every rank owns a staging buffer in torch symmetric memory (so every GPU
    holds device pointers to every rank's copy) and a full-size local output
    [M, 1, L].  One launch per call per rank computes this rank's rows and
    sends every result, as one self-validating 64-bit line (epoch, fp16), to
    every rank's staging buffer over NVLink (``nvfp4_gemv_allgather``); each
    CTA then copies its slice of the lines into the output once they carry this
    call's epoch, so the launch returns with all ranks' rows present.  No NCCL
    call and no fence on the data path.  The staging buffers are reused across
    calls with a running epoch, so one instance serves one fixed shape.
    """

    def __init__(self, M: int, K: int, L: int, group=None, device=None, device_epoch: bool = False):
        """device_epoch=True keeps the call count on the GPU, so calls can be
        captured in a CUDA graph and replayed."""
        import ctypes
        import torch.distributed._symmetric_memory as symm
        self.device_epoch = device_epoch
        self.M, self.K, self.L = M, K, L
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("FusedShardedGemv supports up to 8 ranks")
        # even boundaries: with an even M two results travel per 64-bit line
        self.lo, self.hi = row_split(M, self.world, self.rank, align=2)
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.out_flat = torch.empty(L * M, dtype=torch.float16, device=dev)
        # 64 control words, then one 64-bit line per output element
        self.stage = symm.empty(64 + 2 * M * L, dtype=torch.int32, device=dev)
        self.stage.zero_()
        torch.cuda.synchronize(dev)
        self._h_stage = symm.rendezvous(self.stage, self.group.group_name)
        self._peer_stage = (ctypes.c_void_p * self.world)(*self._h_stage.buffer_ptrs)
        self.epoch = 0
        dist.barrier(self.group)

    def out(self) -> torch.Tensor:
        """[M, 1, L] view of this rank's copy of the full output."""
        return self.out_flat.view(self.L, 1, self.M).permute(2, 1, 0)

    def barrier(self, timeout_ms: int = 10000) -> None:
        """Device-side barrier over this instance's staging buffers (each rank
        signals every peer over NVLink and waits for all), enqueued on the
        current stream: ranks leave it within a peer round trip of each other,
        which lines their next launches up far tighter than a collective does.
        Bounded by timeout_ms."""
        self._h_stage.barrier(channel=0, timeout_ms=timeout_ms)

    def stamps(self) -> tuple[int, int, int]:
        """%globaltimer (ns) of the last call on this rank: launch start, CTA 0
        having sent its rows, last CTA holding its slice of the output."""
        w = self.stage[32:38].cpu().numpy().view("uint32").astype("uint64")
        return tuple(int(w[2 * i]) | (int(w[2 * i + 1]) << 32) for i in range(3))

    def __call__(self, a_rows, b, sfa_rows, sfb) -> torch.Tensor:
        from . import _lib
        self.epoch = 0 if self.device_epoch else ((self.epoch + 1) & 0xFFFFFFFF or 1)
        sa, sb, ssa, ssb = a_rows.stride(), b.stride(), sfa_rows.stride(), sfb.stride()
        _lib.check(_lib.lib().nvfp4_gemv_allgather(
            a_rows.data_ptr(), b.data_ptr(), sfa_rows.data_ptr(), sfb.data_ptr(),
            self.hi - self.lo, self.K, self.L, sa[0], sa[2], sb[2], ssa[0], ssa[2], ssb[2],
            self.out_flat.data_ptr(), 1, self.M, self.lo, self.M, self._peer_stage, self.world, self.rank,
            self.epoch, torch.cuda.current_stream().cuda_stream))
        return self.out()
