"""Page-range sharded selection over the ranks of a torch.distributed group.

One history of `total_pages` pages per layer is split into contiguous page
ranges, one per rank; each rank holds the K of its range in its own HBM. A
decode step on every rank (include/kvm_recall.h, "page-range sharding"):

  1. local page LSE + local softmax statistics           kvm_shard_score_partial
  2. all-gather of the statistics, merge to global ones   kvm_shard_merge_stats
  3. local page masses under the global statistics        kvm_shard_score_finish
  4. local top-B candidates (B = budget - keep pages)     kvm_shard_candidates
  5. all-gather of the candidates, global top-k           kvm_shard_merge

The collectives are two plain all-gathers of small tensors per step (the
statistics; the candidates' scores and ids side by side), NCCL over NVLink on
GPUs; every rank ends with the same selection, equal to a top-k over the
whole row. The compute steps are injected (`ShardCompute`), so the exchange
logic can run with CPU stand-ins on gloo ranks.
"""
from __future__ import annotations

import ctypes as C
import math
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

    def page_lse(self, desc, q, k, geo: ShardGeometry) -> torch.Tensor:
        lse = torch.empty((geo.layers, geo.rows, geo.q_heads, geo.local_pages), dtype=torch.float32,
                          device=f"cuda:{self.ctx.device}")
        A.check(self.lib.kvm_shard_page_lse(self.ctx.h, C.byref(desc), C.byref(q), C.byref(k), geo.page0,
                                            geo.local_pages, lse.data_ptr(), self._s()), "kvm_shard_page_lse")
        return lse

    def mass_from_lse(self, desc, geo: ShardGeometry, lse: torch.Tensor) -> torch.Tensor:
        mass = torch.empty((geo.sel_rows, geo.total_pages), dtype=torch.float32, device=lse.device)
        A.check(self.lib.kvm_page_mass_from_lse(self.ctx.h, C.byref(desc), geo.rows, lse.data_ptr(), None,
                                                mass.data_ptr(), self._s()), "kvm_page_mass_from_lse")
        return mass

    def select_topk(self, mass: torch.Tensor, keep: Sequence[int], budget: int):
        ids = torch.zeros((mass.shape[0], budget), dtype=torch.int32, device=mass.device)
        n = torch.zeros((mass.shape[0],), dtype=torch.int32, device=mass.device)
        return self.ctx.select_topk(mass, keep, budget, out_ids=ids, out_n=n, stream=torch.cuda.current_stream())

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

    def _all_gather_pair(self, a: torch.Tensor, b: torch.Tensor):
        """All-gathers two tensors in one collective (their bytes side by side)."""
        if self.world == 1:
            return a.unsqueeze(0).contiguous(), b.unsqueeze(0).contiguous()
        a, b = a.contiguous(), b.contiguous()
        na = a.numel() * a.element_size()
        packed = torch.cat([a.reshape(-1).view(torch.uint8), b.reshape(-1).view(torch.uint8)])
        g = self._all_gather(packed)  # [world][bytes]
        ga = g[:, :na].contiguous().view(a.dtype).view((self.world,) + tuple(a.shape))
        gb = g[:, na:].contiguous().view(b.dtype).view((self.world,) + tuple(b.shape))
        return ga, gb

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
        gs, gi = self._all_gather_pair(cs, ci)
        return self.compute.merge(gs, gi, self.world, geo, keep, kcand, budget)


class LseGatherSelector(ShardedSelector):
    """Sharded selection with one collective: every rank all-gathers the page LSE of its
    range (layers x rows x query heads x its pages), lays the ranges side by side and
    finishes the whole rows itself (softmax over all pages, head / row means, top-k) with
    the single-GPU kernels, so every rank holds the unsharded selection. The gathered
    LSE is small (config 2: 48 KiB per layer), so this trades a few KB of NVLink traffic
    for one all-gather and four small kernels fewer than ShardedSelector."""

    def select(self, desc, q, k, geo: ShardGeometry, keep: Sequence[int], budget: int):
        keep = sorted(set(int(x) for x in keep))
        if len(keep) > budget:
            raise A.KvmError(A.ERR_BUDGET_EXCEEDED, "sharded select")
        lse = self.compute.page_lse(desc, q, k, geo)  # [L][R][Hq][local pages]
        full = self._gather_lse(lse, geo)  # [L][R][Hq][total pages]
        mass = self.compute.mass_from_lse(desc, geo, full)
        return self.compute.select_topk(mass, keep, budget)

    def _gather_lse(self, lse: torch.Tensor, geo: ShardGeometry) -> torch.Tensor:
        if self.world == 1:
            return lse.contiguous()
        ranges = page_ranges(geo.total_pages, self.world)
        widest = max(e - b for b, e in ranges)
        head = lse.shape[:-1]
        flat = lse.reshape(-1)
        if lse.shape[-1] != widest:  # equal-sized slices for the collective
            pad = torch.empty(math.prod(head) * widest, dtype=lse.dtype, device=lse.device)
            pad[: flat.numel()].copy_(flat)
            flat = pad
        g = self._all_gather(flat)  # [world][slice]
        if all(e - b == widest for b, e in ranges):
            return g.view((self.world,) + tuple(head) + (widest,)).movedim(0, -2).reshape(
                tuple(head) + (geo.total_pages,)).contiguous()
        full = torch.empty(tuple(head) + (geo.total_pages,), dtype=lse.dtype, device=lse.device)
        for w, (b, e) in enumerate(ranges):
            full[..., b:e].copy_(g[w, : flat.numel() // widest * (e - b)].view(tuple(head) + (e - b,)))
        return full


class ShardedRecall:
    """A whole decode-step recall over a page-range partition: selection and stage-in.

    The step is cut into layer chunks, pipelined as in kvm_recall_step. Per chunk, on
    every rank: the sharded selection of the chunk's layers (a ShardedSelector or
    LseGatherSelector), the residency plan of those rows on this rank's copy of the pool
    (every rank plans the same merged selection with the same deterministic kernel, so
    the copies stay identical without a collective), then, on a side stream, the
    gather of the planned restores that lie in this rank's page range, from this rank's
    pinned records over its own PCIe link into the decode rank's paged cache (through a
    peer mapping of it on the other ranks: NVLink). The gather of chunk i overlaps the
    scoring of chunk i + 1. The step ends with a one-element all-reduce enqueued after
    the gathers on every rank: when it completes on the decode rank, every rank's pages
    are in its cache.

    pools[i] / layouts[i]: chunk i's residency table (rows = its layers x groups, all
    pages of the history) and stage-in layout (host records of this rank's range,
    destination = the decode rank's cache rows of the chunk)."""

    def __init__(self, selector: ShardedSelector, pools, layouts, chunk_layers, geo: ShardGeometry,
                 stage_ctas: int = 64):
        self.sel = selector
        self.pools, self.layouts = pools, layouts
        self.chunk_layers = chunk_layers  # [(l0, nl)]
        self.geo = geo
        self.stage_ctas = stage_ctas
        dev = torch.device("cuda", selector.compute.ctx.device)
        self.side = torch.cuda.Stream(device=dev)
        self.events = [torch.cuda.Event() for _ in chunk_layers]
        self.flag = torch.ones(1, dtype=torch.int32, device=dev)
        self.graph = None
        self.graph_launches = 0
        self.ids = torch.zeros((geo.sel_rows, 1), dtype=torch.int32, device=dev)
        self.n = torch.zeros((geo.sel_rows,), dtype=torch.int32, device=dev)

    def step(self, desc, q: torch.Tensor, k, keep: Sequence[int], budget: int, *, force_reload: bool = False,
             stage: bool = True):
        """desc: the whole step's kvm_score_desc (global token count); q: [L][R][Hq][D] device
        queries; k: kvm_kcache of this rank's pages for all layers. Returns (ids, n) of all
        selection rows ([L*groups][budget], [L*groups]), identical on every rank. stage=False
        runs the selection alone (same collectives; no residency plan, no stage-in)."""
        from .recall import RecallContext
        g = self.geo
        if self.ids.shape[1] != budget:
            self.ids = torch.zeros((g.sel_rows, budget), dtype=torch.int32, device=self.ids.device)
        main = torch.cuda.current_stream()
        for ci, (l0, nl) in enumerate(self.chunk_layers):
            d = type(desc).from_buffer_copy(desc)
            d.layers = nl
            kc = type(k).from_buffer_copy(k)
            kc.data = k.data + l0 * k.layer_stride
            qd = RecallContext.make_query(q[l0:l0 + nl], q.shape[1])
            geo = ShardGeometry(layers=nl, rows=g.rows, q_heads=g.q_heads, kv_heads=g.kv_heads, groups=g.groups,
                                total_pages=g.total_pages, page0=g.page0, local_pages=g.local_pages)
            ids, n = self.sel.select(d, qd, kc, geo, keep, budget)
            r0, nr = l0 * g.groups, nl * g.groups
            self.ids[r0:r0 + nr].copy_(ids)
            self.n[r0:r0 + nr].copy_(n)
            if not stage:
                continue
            self.pools[ci].plan(ids, n, force_reload=force_reload)
            self.events[ci].record(main)
            self.side.wait_event(self.events[ci])
            self.pools[ci].stage_in_range(self.layouts[ci], g.page0, g.local_pages, ctas=self.stage_ctas,
                                          stream=self.side)
        main.wait_stream(self.side)
        if self.sel.world > 1:
            dist.all_reduce(self.flag, op=dist.ReduceOp.MAX, group=self.sel.group)  # the decode cache is complete
        return self.ids, self.n

    def capture(self, desc, q_static: torch.Tensor, k, keep: Sequence[int], budget: int, *, warmup: int = 2) -> bool:
        """Records one step (queries read from q_static) into a CUDA graph, so that a step
        costs one launch on the host instead of a few dozen kernel launches, library calls
        and collectives. Every rank must call it at the same point; the ranks agree (one
        all-reduce, outside any graph) to use the graphs only if every rank captured one.
        Returns whether replay() is available."""
        ok = 1
        graph = None
        launches0 = self.sel.compute.ctx.launches
        try:
            s = torch.cuda.Stream(device=q_static.device)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(warmup):
                    self.step(desc, q_static, k, keep, budget)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            launches0 = self.sel.compute.ctx.launches
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self.step(desc, q_static, k, keep, budget)
            torch.cuda.synchronize()
        except Exception:
            ok, graph = 0, None
        self.graph_launches = self.sel.compute.ctx.launches - launches0 if graph is not None else 0
        if self.sel.world > 1:
            t = torch.tensor([ok], dtype=torch.int32, device=q_static.device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.sel.group)
            ok = int(t.item())
        self.graph = graph if ok else None
        return self.graph is not None

    def replay(self):
        """One recorded step (capture() first; refresh q_static before each)."""
        self.graph.replay()
        return self.ids, self.n

    def release(self) -> None:
        """Drops the recorded graph (before the process group is destroyed)."""
        self.graph = None
