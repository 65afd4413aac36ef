"""Page-range sharded selection over the ranks of a torch.distributed group.

One history of `total_pages` pages per layer is split into contiguous page
ranges, one per rank; each rank holds the K of its range in its own HBM. A
decode step on every rank (include/kvm_recall.h, "page-range sharding"):

  1. local page LSE + local softmax statistics           kvm_shard_score_partial
  2. all-gather of the statistics, merge to global ones   kvm_shard_merge_stats
  3. local page masses under the global statistics        kvm_shard_score_finish
  4. local top-B candidates (B = budget - keep pages)     kvm_shard_candidates
  5. all-gather of the candidates, global top-k           kvm_shard_merge

The collectives are plain all-gathers of small tensors (NCCL over NVLink on
GPUs); every rank ends with the same selection, equal to a top-k over the
whole row. The compute steps are injected (`ShardCompute`), so the exchange
logic can run with CPU stand-ins on gloo ranks.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.distributed as dist

from . import _abi as A


def page_ranges(total_pages: int, world: int):
    """Contiguous page range [begin, end) of every rank (sizes differ by at most one)."""
    base, extra = divmod(total_pages, world)
    out, b = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((b, b + n))
        b += n
    return out


@dataclass
class ShardGeometry:
    layers: int
    rows: int
    q_heads: int
    kv_heads: int
    groups: int
    total_pages: int
    page0: int
    local_pages: int

    @property
    def stat_count(self) -> int:
        return self.layers * self.rows * self.q_heads

    @property
    def sel_rows(self) -> int:
        return self.layers * self.groups


class ShardCompute:
    """The five per-rank compute steps on this library's CUDA kernels."""

    def __init__(self, ctx):
        self.ctx = ctx
        self.lib = ctx.lib

    def _s(self):
        return torch.cuda.current_stream().cuda_stream

    def partial(self, desc, q, k, geo: ShardGeometry) -> torch.Tensor:
        stats = torch.empty((geo.stat_count, 2), dtype=torch.float32, device=f"cuda:{self.ctx.device}")
        A.check(self.lib.kvm_shard_score_partial(self.ctx.h, C.byref(desc), C.byref(q), C.byref(k), geo.page0,
                                                 geo.local_pages, stats.data_ptr(), self._s()),
                "kvm_shard_score_partial")
        return stats

    def merge_stats(self, gathered: torch.Tensor, world: int, geo: ShardGeometry) -> torch.Tensor:
        out = torch.empty((geo.stat_count, 2), dtype=torch.float32, device=gathered.device)
        A.check(self.lib.kvm_shard_merge_stats(self.ctx.h, gathered.data_ptr(), world, geo.stat_count,
                                               out.data_ptr(), self._s()), "kvm_shard_merge_stats")
        return out

    def finish(self, desc, geo: ShardGeometry, global_stats: torch.Tensor) -> torch.Tensor:
        mass = torch.empty((geo.sel_rows, geo.local_pages), dtype=torch.float32, device=global_stats.device)
        A.check(self.lib.kvm_shard_score_finish(self.ctx.h, C.byref(desc), geo.rows, geo.local_pages,
                                                global_stats.data_ptr(), None, mass.data_ptr(), self._s()),
                "kvm_shard_score_finish")
        return mass

    def candidates(self, mass: torch.Tensor, geo: ShardGeometry, keep: Sequence[int], k: int):
        cs = torch.empty((geo.sel_rows, k), dtype=torch.float32, device=mass.device)
        ci = torch.empty((geo.sel_rows, k), dtype=torch.int32, device=mass.device)
        kp = (C.c_uint32 * max(1, len(keep)))(*keep)
        A.check(self.lib.kvm_shard_candidates(self.ctx.h, mass.data_ptr(), geo.sel_rows, geo.local_pages,
                                              mass.stride(0), geo.page0, kp, len(keep), k, cs.data_ptr(),
                                              ci.data_ptr(), self._s()), "kvm_shard_candidates")
        return cs, ci

    def merge(self, cs: torch.Tensor, ci: torch.Tensor, world: int, geo: ShardGeometry, keep: Sequence[int],
              k: int, budget: int):
        ids = torch.zeros((geo.sel_rows, budget), dtype=torch.int32, device=cs.device)
        n = torch.zeros((geo.sel_rows,), dtype=torch.int32, device=cs.device)
        kp = (C.c_uint32 * max(1, len(keep)))(*keep)
        A.check(self.lib.kvm_shard_merge(self.ctx.h, cs.data_ptr(), ci.data_ptr(), world, geo.sel_rows, k, kp,
                                         len(keep), budget, ids.data_ptr(), n.data_ptr(), budget, self._s()),
                "kvm_shard_merge")
        return ids, n


class ShardedSelector:
    """Runs the sharded decode-step selection of this rank inside `group`."""

    def __init__(self, compute, group: Optional[dist.ProcessGroup] = None):
        self.compute = compute
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def _all_gather(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t.unsqueeze(0).contiguous()
        t = t.contiguous()
        if dist.get_backend(self.group) == "nccl":
            out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t, group=self.group)
        return torch.stack(parts)

    def select(self, desc, q, k, geo: ShardGeometry, keep: Sequence[int], budget: int):
        """Returns (ids [sel_rows][budget] int32, n [sel_rows] int32), identical on every rank."""
        keep = sorted(set(int(x) for x in keep))
        if len(keep) > budget:
            raise A.KvmError(A.ERR_BUDGET_EXCEEDED, "sharded select")
        kcand = max(1, budget - len(keep))
        stats = self.compute.partial(desc, q, k, geo)
        global_stats = self.compute.merge_stats(self._all_gather(stats), self.world, geo)
        mass = self.compute.finish(desc, geo, global_stats)
        cs, ci = self.compute.candidates(mass, geo, keep, kcand)
        gs, gi = self._all_gather(cs), self._all_gather(ci)
        return self.compute.merge(gs, gi, self.world, geo, keep, kcand, budget)
