"""Host-side API over the C ABI (``include/kvm_recall.h``).

Two layers:

* ``RecallContext`` / ``ResidencyPool`` — direct wrappers of the C entry
  points, taking device tensors (torch is used only to own device memory and
  streams) and returning device tensors;
* ``AttentionCuda``, ``PageSoftmaxCuda`` and ``pick_scored_blocks`` — mirrors
  of the reference's interfaces for this path, with the same argument meaning
  and error behaviour, so callers and tests read like the reference's own:
  ``llama_kvmem_attention_cuda::score`` (src/adapter/llama-kvmem-attention-cuda.h:9-18),
  ``kvmem::PageSoftmaxCuda`` (kvmem/include/kvmem/page_softmax_cuda.hpp:10-31) and
  ``KvMemStore::pick_scored_blocks`` (kvmem/src/host/kvmem_store.cpp:418-451).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _abi as A

_TORCH_QTYPE = {torch.float32: A.F32, torch.float16: A.F16, torch.bfloat16: A.BF16}


def _stream_ptr(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def row_bytes(ktype: int, dim: int) -> int:
    return int(A.load().kvm_row_bytes(ktype, dim))


class RecallContext:
    """One kvm_ctx: device, status word, scoring workspace, stage-in stream."""

    def __init__(self, device: int = 0):
        self.lib = A.load()
        self.device = device
        h = C.c_void_p()
        A.check(self.lib.kvm_ctx_create(device, C.byref(h)), "kvm_ctx_create")
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.kvm_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- status / workspace ------------------------------------------------
    def status(self, stream=None) -> int:
        return int(self.lib.kvm_ctx_status(self.h, _stream_ptr(stream)))

    def check_status(self, where: str = "device", stream=None) -> None:
        A.check(self.status(stream), where)

    @property
    def launches(self) -> int:
        return int(self.lib.kvm_ctx_launches(self.h))

    def bind_workspace(self, tensor: torch.Tensor) -> None:
        A.check(self.lib.kvm_ctx_bind_workspace(self.h, tensor.data_ptr(), tensor.numel() * tensor.element_size()),
                "kvm_ctx_bind_workspace")

    def device_bytes(self) -> int:
        return int(self.lib.kvm_ctx_device_bytes(self.h))

    # -- descriptors -------------------------------------------------------
    @staticmethod
    def make_desc(*, layers, q_heads, kv_heads, head_dim, tokens, page_tokens, groups=1, scale=0.0, softcap=0.0,
                  mask: Optional[torch.Tensor] = None, mask_row_stride: int = 0) -> A.ScoreDesc:
        d = A.ScoreDesc()
        d.layers, d.q_heads, d.kv_heads, d.head_dim = layers, q_heads, kv_heads, head_dim
        d.tokens, d.page_tokens, d.groups = tokens, page_tokens, groups
        d.scale, d.softcap = scale, softcap
        if mask is not None:
            d.mask = mask.data_ptr()
            d.mask_type = _TORCH_QTYPE[mask.dtype]
            d.mask_row_stride = mask_row_stride or mask.stride(0) * mask.element_size()
        return d

    @staticmethod
    def make_query(q: torch.Tensor, rows: int, *, strides=None, data_ptr: Optional[int] = None,
                   row_ids: Optional[Sequence[int]] = None, row_count: int = 0) -> A.Query:
        """q dense [layers][rows][heads][dim] unless strides=(layer, row, head) bytes.
        row_ids: score only these rows of the tensor (the reference's sampled `rows`);
        `rows` is then len(row_ids) and row_count the rows the tensor holds."""
        qq = A.Query()
        qq.data = data_ptr if data_ptr is not None else q.data_ptr()
        qq.type = _TORCH_QTYPE[q.dtype]
        qq.rows = rows
        es = q.element_size()
        if strides is None:
            L, R, H, D = q.shape
            strides = (R * H * D * es, H * D * es, D * es)
        qq.layer_stride, qq.row_stride, qq.head_stride = strides
        if row_ids is not None:
            ids = (C.c_uint32 * max(1, len(row_ids)))(*row_ids)
            qq.row_ids = C.cast(ids, C.POINTER(C.c_uint32))
            qq._ids = ids  # keeps the host list alive with the descriptor
            qq.rows = len(row_ids)
            qq.row_count = row_count or (q.shape[1] if q.dim() == 4 else 0)
        return qq

    @staticmethod
    def make_kcache(k: torch.Tensor, ktype: int, *, kv_heads: int, head_dim: int, capacity_tokens: int,
                    layer_stride: Optional[int] = None, data_ptr: Optional[int] = None) -> A.KCache:
        """k: device bytes holding [layers][capacity_tokens][kv_heads] rows of ktype."""
        kc = A.KCache()
        kc.data = data_ptr if data_ptr is not None else k.data_ptr()
        kc.type = ktype
        rb = row_bytes(ktype, head_dim)
        kc.head_stride = rb
        kc.token_stride = rb * kv_heads
        kc.layer_stride = layer_stride if layer_stride is not None else rb * kv_heads * capacity_tokens
        kc.capacity_tokens = capacity_tokens
        return kc

    # -- entry points ------------------------------------------------------
    def score_pages(self, desc: A.ScoreDesc, q: A.Query, k: A.KCache, *, want_rows=True, want_mean=True,
                    out_rows: Optional[torch.Tensor] = None, out_mean: Optional[torch.Tensor] = None, stream=None):
        pages = -(-desc.tokens // desc.page_tokens)
        dev = torch.device("cuda", self.device)
        if want_rows and out_rows is None:
            out_rows = torch.empty((desc.layers, desc.groups, q.rows, pages), dtype=torch.float32, device=dev)
        if want_mean and out_mean is None:
            out_mean = torch.empty((desc.layers, desc.groups, pages), dtype=torch.float32, device=dev)
        rc = self.lib.kvm_score_pages(self.h, C.byref(desc), C.byref(q), C.byref(k),
                                      out_rows.data_ptr() if out_rows is not None else None,
                                      out_mean.data_ptr() if out_mean is not None else None, _stream_ptr(stream))
        A.check(rc, "kvm_score_pages")
        return out_rows, out_mean

    def prefill_attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, base: int,
                          sample_rows: Sequence[int] = (), page_tokens: int = 64, pages: Optional[int] = None,
                          scale: float = 0.0, out: Optional[torch.Tensor] = None,
                          page_lse: Optional[torch.Tensor] = None, stream=None):
        """Causal prompt attention with the page LSE of the sampled rows captured in the same pass
        (kvm_prefill_attention; the engine's causal_softmax_attention_with_page_lse).

        q: [width][q_heads][head_dim] fp16 / bf16 prompt rows at positions base .. base + width - 1;
        k, v: [capacity][kv_heads][head_dim] cache views holding keys 0 .. base + width - 1.
        Returns (out [width][q_heads][head_dim], page_lse [samples][q_heads][pages] or None)."""
        assert q.dim() == 3 and k.dim() == 3 and v.dim() == 3 and q.dtype == k.dtype == v.dtype
        width, hq, dim = q.shape
        cap, hkv, _ = k.shape
        t = _TORCH_QTYPE[q.dtype]
        d = A.PrefillDesc()
        d.q_heads, d.kv_heads, d.head_dim, d.type = hq, hkv, dim, t
        d.base, d.width, d.scale = base, width, scale
        rows = list(sample_rows)
        d.samples = len(rows)
        d.page_tokens = page_tokens
        d.pages = pages if pages is not None else -(-(base + width) // page_tokens)
        ids = (C.c_uint32 * max(1, len(rows)))(*rows)
        d.sample_rows = C.cast(ids, C.POINTER(C.c_uint32))
        if out is None:
            out = torch.empty_like(q)
        if rows and page_lse is None:
            page_lse = torch.empty((len(rows), hq, d.pages), dtype=torch.float32, device=q.device)
        es = q.element_size()

        def view(x: torch.Tensor) -> A.KCache:
            kc = A.KCache()
            kc.data, kc.type = x.data_ptr(), t
            kc.token_stride, kc.head_stride = x.stride(0) * es, x.stride(1) * es
            kc.layer_stride, kc.capacity_tokens = 0, x.shape[0]
            return kc

        kc, vc = view(k), view(v)
        rc = self.lib.kvm_prefill_attention(self.h, C.byref(d), q.data_ptr(), q.stride(0) * es, q.stride(1) * es,
                                            C.byref(kc), C.byref(vc), out.data_ptr(), out.stride(0) * es,
                                            out.stride(1) * es, page_lse.data_ptr() if rows else None,
                                            _stream_ptr(stream))
        A.check(rc, "kvm_prefill_attention")
        return out, (page_lse if rows else None)

    def page_mass_from_lse(self, desc: A.ScoreDesc, rows: int, lse: torch.Tensor, *, want_rows=True,
                           want_mean=True, stream=None):
        """Whole-history page LSE [layers][rows][q_heads][pages] -> (mass_rows, mass_mean) as score_pages."""
        pages = -(-desc.tokens // desc.page_tokens)
        dev = lse.device
        out_rows = torch.empty((desc.layers, desc.groups, rows, pages), dtype=torch.float32, device=dev) \
            if want_rows else None
        out_mean = torch.empty((desc.layers, desc.groups, pages), dtype=torch.float32, device=dev) \
            if want_mean else None
        rc = self.lib.kvm_page_mass_from_lse(self.h, C.byref(desc), rows, lse.data_ptr(),
                                             out_rows.data_ptr() if out_rows is not None else None,
                                             out_mean.data_ptr() if out_mean is not None else None,
                                             _stream_ptr(stream))
        A.check(rc, "kvm_page_mass_from_lse")
        return out_rows, out_mean

    def select_topk(self, scores: torch.Tensor, keep: Sequence[int], budget: int, *, signed: bool = False,
                    out_ids: Optional[torch.Tensor] = None, out_n: Optional[torch.Tensor] = None, stream=None):
        """scores [nrows][pages] f32 on the device -> (ids [nrows][min(budget,pages)], n [nrows])."""
        assert scores.dtype == torch.float32 and scores.dim() == 2
        nrows, pages = scores.shape
        width = min(budget, pages)
        if out_ids is None:
            out_ids = torch.zeros((nrows, width), dtype=torch.int32, device=scores.device)
        if out_n is None:
            out_n = torch.zeros((nrows,), dtype=torch.int32, device=scores.device)
        kp = (C.c_uint32 * max(1, len(keep)))(*keep)
        rc = self.lib.kvm_select_topk(self.h, scores.data_ptr(), nrows, pages, scores.stride(0), kp, len(keep),
                                      budget, int(signed), out_ids.data_ptr(), out_n.data_ptr(), out_ids.stride(0),
                                      _stream_ptr(stream))
        A.check(rc, "kvm_select_topk")
        return out_ids, out_n

    def select_topk_media(self, scores: torch.Tensor, keep: Sequence[int], budget: int, *, block_tokens: int,
                          media_ranges: Sequence[tuple], signed: bool = False, stream=None):
        """select_topk with media groups (KvMemStore::pick_scored_blocks with the store's
        media ranges, token [begin, end) pairs; pages of block_tokens tokens)."""
        assert scores.dtype == torch.float32 and scores.dim() == 2
        nrows, pages = scores.shape
        width = min(budget, pages)
        out_ids = torch.zeros((nrows, width), dtype=torch.int32, device=scores.device)
        out_n = torch.zeros((nrows,), dtype=torch.int32, device=scores.device)
        kp = (C.c_uint32 * max(1, len(keep)))(*keep)
        flat = [int(x) for r in media_ranges for x in r]
        rg = (C.c_uint32 * max(1, len(flat)))(*flat)
        rc = self.lib.kvm_select_topk_media(self.h, scores.data_ptr(), nrows, pages, scores.stride(0), kp, len(keep),
                                            budget, int(signed), block_tokens, rg, len(media_ranges),
                                            out_ids.data_ptr(), out_n.data_ptr(), out_ids.stride(0),
                                            _stream_ptr(stream))
        A.check(rc, "kvm_select_topk_media")
        return out_ids, out_n

    def restore_k(self, ktype: int, items: Sequence[tuple], *, n_head: int, head_dim: int, n_rot: int = 0,
                  theta: Optional[Sequence[float]] = None, nrot: int = 0, stream=None) -> None:
        """items: (src_ptr, dst_ptr, tokens, pos0) -> kvm_restore_k (raw-K restore transform)."""
        arr = (A.RestoreItem * max(1, len(items)))()
        for i, (src, dst, tokens, pos0) in enumerate(items):
            arr[i].src, arr[i].dst, arr[i].tokens, arr[i].pos0 = src, dst, tokens, pos0
        th = (C.c_float * max(1, n_rot // 2))(*(list(theta or [])[: n_rot // 2]))
        rc = self.lib.kvm_restore_k(self.h, ktype, arr, len(items), n_head, head_dim, n_rot, th, nrot,
                                    _stream_ptr(stream))
        A.check(rc, "kvm_restore_k")

    @staticmethod
    def make_graph(graph: dict):
        """kvm_graph from dict(block, accepted, completed, rows=[(source, samples, [(target, mass), ...])],
        spans=None | [(begin, end, end_known)]); returns (struct, keepalive)."""
        rows = graph.get("rows", [])
        edges = [e for r in rows for e in r[2]]
        spans = graph.get("spans")
        ra = (A.GraphRow * max(1, len(rows)))()
        ea = (A.GraphEdge * max(1, len(edges)))()
        sa = (A.GraphSpan * max(1, len(spans or [])))()
        off = 0
        for i, (src, samples, es) in enumerate(rows):
            ra[i].source, ra[i].samples, ra[i].edge_begin, ra[i].edge_count = src, samples, off, len(es)
            off += len(es)
        for i, (tgt, mass) in enumerate(edges):
            ea[i].target, ea[i].mass = tgt, mass
        for i, (b, e, known) in enumerate(spans or []):
            sa[i].begin, sa[i].end, sa[i].end_known = b, e, int(bool(known))
        g = A.Graph()
        g.block_tokens, g.has_messages = graph["block"], int(spans is not None)
        g.accepted_through, g.completed_through = graph["accepted"], graph["completed"]
        g.rows, g.nrows, g.edges, g.nedges = ra, len(rows), ea, len(edges)
        g.spans, g.nspans = sa, len(spans or [])
        return g, (ra, ea, sa)

    def propagate_scores(self, raw: torch.Tensor, starts: Sequence[int], transport_mask: Sequence[int],
                         accepted: int, graph: dict, *, alpha: float = 0.2, cross: float = 0.25,
                         out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """raw [n] f32 on the device -> propagated scores [n] f32 (kvm_propagate_scores)."""
        n = raw.numel()
        if out is None:
            out = torch.empty_like(raw)
        st = (C.c_uint64 * max(1, n))(*starts)
        tm = (C.c_uint8 * max(1, n))(*[1 if x else 0 for x in transport_mask])
        g, keep = self.make_graph(graph)
        rc = self.lib.kvm_propagate_scores(self.h, raw.data_ptr(), n, st, tm, accepted, C.byref(g), alpha, cross,
                                           out.data_ptr(), _stream_ptr(stream))
        A.check(rc, "kvm_propagate_scores")
        return out

    def lrfu_preview(self, scores: torch.Tensor, prev: Optional[torch.Tensor], *, lam: float = 0.5,
                     fraction: float = 0.9, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """scores [n] f32, prev [n_prev] f32 (committed history, device) -> candidate [n] f32."""
        n = scores.numel()
        if out is None:
            out = torch.empty_like(scores)
        n_prev = 0 if prev is None else prev.numel()
        rc = self.lib.kvm_lrfu_preview(self.h, scores.data_ptr(), n, prev.data_ptr() if n_prev else None, n_prev,
                                       lam, fraction, out.data_ptr(), _stream_ptr(stream))
        A.check(rc, "kvm_lrfu_preview")
        return out

    def meank_add(self, k: A.KCache, sums: torch.Tensor, counts: torch.Tensor, *, tok0: int, n: int,
                  page_tokens: int, kv_heads: int, head_dim: int, stream=None) -> None:
        """Adds tokens [tok0, tok0 + n) of every layer of `k` into the per-page sums
        [L][P][Hkv*D] f32 and their count into counts [P] (int32 tensor, read as u32)."""
        L, P, E = sums.shape
        if E != kv_heads * head_dim or counts.numel() < P:
            raise A.KvmError(A.ERR_INVALID_ARGUMENT, "meank_add: table shape")
        rc = self.lib.kvm_meank_add(self.h, C.byref(k), L, kv_heads, head_dim, tok0, n, page_tokens,
                                    sums.data_ptr(), P, counts.data_ptr(), _stream_ptr(stream))
        A.check(rc, "kvm_meank_add")

    def meank_score(self, sums: torch.Tensor, counts: torch.Tensor, q: torch.Tensor, layer_rows: Sequence[int],
                    score_mask: Sequence[int], *, q_heads: int, kv_heads: int, head_dim: int, aggregation: int = 0,
                    scale: float = 0.0, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """sums [L][P][Hkv*D] f32, counts [P] u32 (int32 tensor), q [L][R][Hq*D] f32 -> out [P] f32."""
        L, P, _ = sums.shape
        R = q.shape[1]
        if out is None:
            out = torch.empty((P,), dtype=torch.float32, device=sums.device)
        lr = (C.c_uint32 * L)(*layer_rows)
        sm = (C.c_uint8 * P)(*[1 if x else 0 for x in score_mask])
        rc = self.lib.kvm_meank_score(self.h, sums.data_ptr(), counts.data_ptr(), q.data_ptr(), lr, L, R, q_heads,
                                      kv_heads, head_dim, P, sm, aggregation, scale, out.data_ptr(),
                                      _stream_ptr(stream))
        A.check(rc, "kvm_meank_score")
        return out

    def layerwise_accumulate(self, tile: torch.Tensor, score_mask: torch.Tensor, accum: torch.Tensor, *,
                             halves: int = 1, keep_halves: bool = False, stream=None) -> None:
        """kvm_layerwise_accumulate: tile f32 [pages * halves], score_mask u8 [pages],
        accum f64 [pages * (2 if keep_halves else 1)] (all device)."""
        pages = score_mask.numel()
        A.check(self.lib.kvm_layerwise_accumulate(self.h, tile.data_ptr(), pages, halves, int(keep_halves),
                                                  score_mask.data_ptr(), accum.data_ptr(), _stream_ptr(stream)),
                "kvm_layerwise_accumulate")

    def layerwise_finish(self, accum: torch.Tensor, pages: int, *, keep_halves: bool = False,
                         out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """kvm_layerwise_finish -> scores f32 [pages] (device)."""
        if out is None:
            out = torch.empty((pages,), dtype=torch.float32, device=accum.device)
        A.check(self.lib.kvm_layerwise_finish(self.h, accum.data_ptr(), pages, int(keep_halves), out.data_ptr(),
                                              _stream_ptr(stream)), "kvm_layerwise_finish")
        return out

    def stagein_copies(self, ops: Sequence[tuple], ctas: int = 0, stream=None) -> None:
        arr = (A.Copy * max(1, len(ops)))()
        for i, (src, dst, nbytes) in enumerate(ops):
            arr[i].src, arr[i].dst, arr[i].bytes = src, dst, nbytes
        A.check(self.lib.kvm_stagein_copies(self.h, arr, len(ops), ctas, _stream_ptr(stream)), "kvm_stagein_copies")

    def wait(self, timeout_s: float = 30.0, stream=None) -> None:
        A.check(self.lib.kvm_stagein_wait(self.h, _stream_ptr(stream), int(timeout_s * 1e6)), "kvm_stagein_wait")

    def recall_step(self, desc: A.ScoreDesc, q: A.Query, k: A.KCache, keep: Sequence[int], budget: int, *,
                    mass_mean: torch.Tensor, sel_ids: torch.Tensor, sel_n: torch.Tensor,
                    pool: Optional["ResidencyPool"] = None, layout: Optional[A.StageLayout] = None,
                    chunks: int = 0, stage_ctas: int = 0, force_reload: bool = False, first_layers: int = 0,
                    stream=None) -> None:
        st = A.StepDesc()
        st.score = C.pointer(desc)
        st.q = C.pointer(q)
        st.k = C.pointer(k)
        kp = (C.c_uint32 * max(1, len(keep)))(*keep)
        st.keep = C.cast(kp, C.POINTER(C.c_uint32))
        st.nkeep, st.budget, st.chunks, st.stage_ctas = len(keep), budget, chunks, stage_ctas
        st.force_reload = int(force_reload)
        st.first_layers = first_layers
        rc = self.lib.kvm_recall_step(self.h, C.byref(st), pool.h if pool is not None else None,
                                      C.byref(layout) if layout is not None else None, mass_mean.data_ptr(),
                                      sel_ids.data_ptr(), sel_n.data_ptr(), _stream_ptr(stream))
        A.check(rc, "kvm_recall_step")


class ResidencyPool:
    """Device residency table (kvm_pool) for `rows` selections over `pages` pages and `slots` slots."""

    def __init__(self, ctx: RecallContext, rows: int, pages: int, slots: int):
        self.ctx, self.rows, self.pages, self.slots = ctx, rows, pages, slots
        h = C.c_void_p()
        A.check(ctx.lib.kvm_pool_create(ctx.h, rows, pages, slots, C.byref(h)), "kvm_pool_create")
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.ctx.lib.kvm_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, stream=None) -> None:
        A.check(self.ctx.lib.kvm_pool_reset(self.h, _stream_ptr(stream)), "kvm_pool_reset")

    def plan(self, sel_ids: torch.Tensor, sel_n: torch.Tensor, *, force_reload=False, stream=None):
        n_restore = torch.zeros((self.rows,), dtype=torch.int32, device=sel_ids.device)
        n_evict = torch.zeros((self.rows,), dtype=torch.int32, device=sel_ids.device)
        rc = self.ctx.lib.kvm_plan_residency(self.ctx.h, self.h, sel_ids.data_ptr(), sel_n.data_ptr(),
                                             sel_ids.stride(0), int(force_reload), n_restore.data_ptr(),
                                             n_evict.data_ptr(), _stream_ptr(stream))
        A.check(rc, "kvm_plan_residency")
        return n_restore, n_evict

    def stage_in(self, layout: A.StageLayout, ctas: int = 0, stream=None) -> None:
        A.check(self.ctx.lib.kvm_stagein_pool(self.ctx.h, self.h, C.byref(layout), ctas, _stream_ptr(stream)),
                "kvm_stagein_pool")

    def stage_in_range(self, layout: A.StageLayout, page0: int, page_count: int, ctas: int = 0,
                       stream=None) -> None:
        """kvm_shard_stagein: the planned restores of pages [page0, page0 + page_count) from
        this rank's records (layout.host_base starts at page0) into layout.dev_base, which
        may be a peer mapping of the decode GPU's cache (ipc_open)."""
        A.check(self.ctx.lib.kvm_shard_stagein(self.ctx.h, self.h, C.byref(layout), page0, page_count, ctas,
                                               _stream_ptr(stream)), "kvm_shard_stagein")

    def read(self, stream=None):
        import numpy as np
        slot_of = np.empty((self.rows, self.pages), np.int32)
        page_of = np.empty((self.rows, self.slots), np.int32)
        rc = self.ctx.lib.kvm_pool_read(self.h, slot_of.ctypes.data, page_of.ctypes.data, _stream_ptr(stream))
        A.check(rc, "kvm_pool_read")
        return slot_of, page_of


class Transfer:
    """A working-set transfer over a ResidencyPool (kvm_transfer): the GPU side of
    kvmem::MemoryTransfer (kvmem/include/kvmem/memory_contract.hpp:171-185). The
    plan goes into a shadow of the pool's tables; start_spill / poll / start_restore /
    publish / abort keep the reference's names and order; failures raise KvmError
    (the reference's MemoryError codes)."""

    def __init__(self, pool: "ResidencyPool", sel_ids: torch.Tensor, sel_n: torch.Tensor, *,
                 force_reload: bool = False, stream=None):
        self.pool, self.lib = pool, pool.ctx.lib
        h = C.c_void_p()
        rc = self.lib.kvm_transfer_prepare(pool.ctx.h, pool.h, sel_ids.data_ptr(), sel_n.data_ptr(),
                                           sel_ids.stride(0), int(force_reload), _stream_ptr(stream), C.byref(h))
        A.check(rc, "kvm_transfer_prepare")
        self.h = h

    def start_spill(self, layout: Optional[A.StageLayout] = None, stale: Optional[torch.Tensor] = None,
                    ctas: int = 0, stream=None) -> None:
        rc = self.lib.kvm_transfer_start_spill(self.h, C.byref(layout) if layout is not None else None,
                                               stale.data_ptr() if stale is not None else None, ctas,
                                               _stream_ptr(stream))
        A.check(rc, "kvm_transfer_start_spill")

    def poll(self) -> str:
        """'Complete' or 'Pending' (TransferStatus); a failed step raises."""
        rc = self.lib.kvm_transfer_poll(self.h)
        if rc == A.ERR_PENDING:
            return "Pending"
        A.check(rc, "kvm_transfer_poll")
        return "Complete"

    def wait(self, timeout_s: float = 30.0) -> None:
        import time
        t0 = time.time()
        while self.poll() == "Pending":
            if time.time() - t0 > timeout_s:
                raise A.KvmError(A.ERR_TIMEOUT, "kvm_transfer_poll")
            time.sleep(0.0005)

    def start_restore(self, layout: A.StageLayout, ctas: int = 0, stream=None) -> None:
        A.check(self.lib.kvm_transfer_start_restore(self.h, C.byref(layout), ctas, _stream_ptr(stream)),
                "kvm_transfer_start_restore")

    def publish(self, stream=None) -> None:
        A.check(self.lib.kvm_transfer_publish(self.h, _stream_ptr(stream)), "kvm_transfer_publish")

    def abort(self, timeout_s: float = 30.0) -> bool:
        """Drains, then drops the transfer; True when the previous view is preserved."""
        kept = C.c_int(0)
        A.check(self.lib.kvm_transfer_abort(self.h, int(timeout_s * 1e6), C.byref(kept)), "kvm_transfer_abort")
        return bool(kept.value)

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.kvm_transfer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StageOut:
    """Double-buffered stage-out (kvm_stageout): device regions gathered into
    two pinned host slots in turn. Method names follow the reference's
    kvmem_stageout_* functions (src/adapter/llama-kvmem-stagein.h:50-55);
    failures raise KvmError instead of returning false / -1."""

    SLAB = 32 << 20  # the reference's slot size
    GATHER_MAX = 8192

    def __init__(self, device: int = 0, slot_bytes: int = SLAB, max_items: int = GATHER_MAX):
        self.lib = A.load()
        self.slot_bytes = slot_bytes
        h = C.c_void_p()
        A.check(self.lib.kvm_stageout_create(device, slot_bytes, max_items, C.byref(h)), "kvm_stageout_create")
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.kvm_stageout_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def enqueue(self, dev_ptr: int, nbytes: int) -> Optional[int]:
        """Queue a device region; its slot offset, or None when the batch is full."""
        off = C.c_uint64()
        rc = self.lib.kvm_stageout_enqueue(self.h, dev_ptr, nbytes, C.byref(off))
        if rc == A.ERR_LENGTH:
            return None
        A.check(rc, "kvm_stageout_enqueue")
        return off.value

    def used(self) -> int:
        return int(self.lib.kvm_stageout_used(self.h))

    def submit(self, ctas: int = 0, stream=None) -> int:
        slot = C.c_int(-1)
        A.check(self.lib.kvm_stageout_submit(self.h, ctas, _stream_ptr(stream), C.byref(slot)), "kvm_stageout_submit")
        return slot.value

    def wait(self, slot: int, timeout_s: float = 30.0) -> None:
        A.check(self.lib.kvm_stageout_wait(self.h, slot, int(timeout_s * 1e6)), "kvm_stageout_wait")

    def slot_view(self, slot: int, offset: int, nbytes: int):
        """numpy uint8 view of bytes [offset, offset + nbytes) of a slot (no copy)."""
        import numpy as np
        base = self.lib.kvm_stageout_slot_base(self.h, slot)
        if not base or offset + nbytes > self.slot_bytes:
            raise ValueError("slot range")
        buf = (C.c_uint8 * nbytes).from_address(base + offset)
        return np.frombuffer(buf, dtype=np.uint8)

    def clear(self) -> None:
        A.check(self.lib.kvm_stageout_clear(self.h), "kvm_stageout_clear")


def ipc_export(t: torch.Tensor) -> bytes:
    """Opaque handle (kvm_ipc_export) naming a device tensor's memory for another process."""
    buf = (C.c_uint8 * A.IPC_HANDLE_BYTES)()
    A.check(A.load().kvm_ipc_export(t.data_ptr(), buf), "kvm_ipc_export")
    return bytes(buf)


def ipc_open(device: int, handle: bytes) -> int:
    """Maps another process's device memory on `device` (peer access enabled); returns the address."""
    buf = (C.c_uint8 * A.IPC_HANDLE_BYTES).from_buffer_copy(handle)
    ptr = C.c_void_p()
    A.check(A.load().kvm_ipc_open(device, buf, C.byref(ptr)), "kvm_ipc_open")
    return int(ptr.value)


def ipc_close(device: int, ptr: int) -> None:
    A.check(A.load().kvm_ipc_close(device, ptr), "kvm_ipc_close")


def stage_layout(planes: Sequence[dict]) -> A.StageLayout:
    """planes: up to two dicts with host_base, host_row_stride, host_page_stride,
    dev_base, dev_row_stride, dev_slot_stride, bytes."""
    L = A.StageLayout()
    L.planes = len(planes)
    for j, p in enumerate(planes):
        L.host_base[j] = p["host_base"]
        L.host_row_stride[j] = p["host_row_stride"]
        L.host_page_stride[j] = p["host_page_stride"]
        L.dev_base[j] = p["dev_base"]
        L.dev_row_stride[j] = p["dev_row_stride"]
        L.dev_slot_stride[j] = p["dev_slot_stride"]
        L.bytes[j] = p["bytes"]
    return L


# ----------------------------------------------------------------------------
# Mirrors of the reference interfaces for this path.
# ----------------------------------------------------------------------------

@dataclass
class TensorView:
    """The parts of a ggml tensor the reference scorer reads: `data` (device
    tensor owning the bytes), element / block `type`, ne[0..2] and byte strides
    nb[1..2] (ggml order: ne0 = head_dim, ne1 = rows or tokens, ne2 = heads)."""
    data: torch.Tensor
    type: int
    ne: tuple
    nb: tuple


class AttentionCuda:
    """Mirror of llama_kvmem_attention_cuda (src/adapter/llama-kvmem-attention-cuda.h:9-18).

    score(q, k, mask, scale, softcap, block, rows) returns masses[len(rows)][pages]
    (mean over all query heads of the page-softmax mass), or None when the
    inputs are outside what the kernel handles (the reference's `false`,
    after which the caller builds its fallback graph). CUDA failures raise.
    """

    def __init__(self, device: int = 0):
        self.ctx = RecallContext(device)

    def score(self, q: TensorView, k: TensorView, mask: Optional[TensorView], scale: float, softcap: float,
              block: int, rows: Sequence[int]):
        D, _, Hq = q.ne[0], q.ne[1], q.ne[2]
        T, Hkv = k.ne[1], k.ne[2]
        if q.type not in (A.F32, A.F16, A.BF16) or D > 256 or D % 32:
            return None
        pages = -(-T // block)
        desc = RecallContext.make_desc(layers=1, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=block,
                                       groups=1, scale=scale, softcap=softcap)
        kc = A.KCache()
        kc.data, kc.type = k.data.data_ptr(), k.type
        kc.layer_stride, kc.token_stride, kc.head_stride = 0, k.nb[1], k.nb[2]
        kc.capacity_tokens = T
        if not rows:
            return []
        # Every sampled row in one call (one pass over K), as the reference's batch.
        qq = A.Query()
        qq.data = q.data.data_ptr()
        qq.type = q.type
        qq.layer_stride, qq.row_stride, qq.head_stride = 0, q.nb[1], q.nb[2]
        ids = (C.c_uint32 * len(rows))(*rows)
        qq.row_ids = C.cast(ids, C.POINTER(C.c_uint32))
        qq.rows, qq.row_count = len(rows), q.ne[1]
        if mask is not None:
            desc.mask = mask.data.data_ptr()
            desc.mask_type = mask.type
            desc.mask_row_stride = mask.nb[1]
        try:
            out_rows, _ = self.ctx.score_pages(desc, qq, kc, want_mean=False)
        except A.KvmError as e:
            if e.code == A.ERR_UNSUPPORTED:
                return None
            raise
        self.ctx.check_status("llama_kvmem_attention_cuda::score")
        return out_rows.view(len(rows), pages).tolist()


class PageSoftmaxCuda:
    """Mirror of kvmem::PageSoftmaxCuda (kvmem/include/kvmem/page_softmax_cuda.hpp:10-31)
    over device-resident per-page K sums.

    score(sums, counts, q, layer_rows, frame, aggregation) -> list of doubles
    over frame pages; frame is the dict form of QueryScoreFrame (score_mask
    selects the softmax domain). Geometry errors raise ValueError
    (std::invalid_argument), a non-finite / FP16-overflowing operand raises
    ValueError, CUDA failures raise RuntimeError.
    """

    def __init__(self, device: int = 0, workspace: Optional[torch.Tensor] = None):
        self.ctx = RecallContext(device)
        if workspace is not None:
            if workspace.data_ptr() % 256:
                raise ValueError("page softmax borrowed workspace is missing, unaligned or too small")
            self.ctx.bind_workspace(workspace)

    def score(self, sums: torch.Tensor, counts: torch.Tensor, q: torch.Tensor, layer_rows: Sequence[int],
              frame: dict, aggregation: int = 0, *, q_heads: int, kv_heads: int, head_dim: int,
              scale: float = 0.0) -> list:
        try:
            out = self.ctx.meank_score(sums, counts, q, layer_rows, frame["score_mask"], q_heads=q_heads,
                                       kv_heads=kv_heads, head_dim=head_dim, aggregation=aggregation, scale=scale)
        except A.KvmError as e:
            if e.code in (A.ERR_INVALID_ARGUMENT, A.ERR_NONFINITE):
                raise ValueError(str(e)) from e
            if e.code == A.ERR_LENGTH:
                raise OverflowError(str(e)) from e
            raise
        return [float(x) for x in out.cpu().double()]

    def device_bytes(self) -> int:
        return self.ctx.device_bytes()


def pick_scored_blocks(ctx: RecallContext, scores: torch.Tensor, mandatory: Sequence[int], budget: int,
                       signed_scores: bool = False) -> list:
    """Mirror of KvMemStore::pick_scored_blocks with candidates = every page of
    the (device f32) score row and no media groups. Raises ValueError for an
    invalid candidate or mandatory page (std::invalid_argument) and
    RuntimeError when mandatory pages exceed the budget (std::runtime_error)."""
    try:
        ids, n = ctx.select_topk(scores.view(1, -1), mandatory, budget, signed=signed_scores)
        ctx.check_status("pick_scored_blocks")
    except A.KvmError as e:
        if e.code in (A.ERR_INVALID_ARGUMENT, A.ERR_NONFINITE):
            raise ValueError(str(e)) from e
        raise RuntimeError(str(e)) from e
    return ids[0, : int(n[0])].tolist()
