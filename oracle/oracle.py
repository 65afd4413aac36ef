"""CPU ORACLE — test infrastructure only.

ctypes wrappers over

* ``oracle/_ref/liboracle.so`` — the plain-C restatement of the reference
  algorithms (``oracle/kvm_oracle.c``), and
* ``oracle/_ref/libkvref.so`` — the reference's own CPU selection code compiled
  from its sources (``oracle/Makefile`` target ``ref``; present only where the
  reference sources were available when it was built), and
* ``oracle/_ref/libkvref_cuda.so`` — the reference's own GPU scorers compiled
  from its sources for sm_100a (target ``refcuda``): the per-token page mass
  ``llama_kvmem_attention_cuda::score`` and the Mean-K ``PageSoftmaxCuda::score``.

Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference
arm may import this module. The product package ``kvmem_b200`` never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
# The reference checkout: $KVM_REFERENCE_SRC, else the sibling directory
# "reference" of the repository root.
REFERENCE_SRC = os.environ.get("KVM_REFERENCE_SRC") or os.path.normpath(
    os.path.join(HERE, os.pardir, os.pardir, "reference"))

F32, F16, BF16, Q8_0, Q4_0, Q5_0 = 0, 1, 2, 3, 4, 5
OK, ERR_INVALID, ERR_RUNTIME = 0, 1, 2

_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")


def build(ref: bool = False) -> None:
    """Compile the C restatement and, with ref=True (and the reference sources
    present), the reference's own CPU selection library."""
    subprocess.check_call(["make", "-s", "-C", HERE], stdout=subprocess.DEVNULL)
    if ref and os.path.isdir(os.path.join(REFERENCE_SRC, "kvmem", "src", "host")):
        subprocess.check_call(["make", "-s", "-j8", "-C", HERE, "ref", f"REF={REFERENCE_SRC}"],
                              stdout=subprocess.DEVNULL)
        if os.path.exists(os.path.join(REFERENCE_SRC, "src", "adapter", "llama-kvmem-attention-cuda.cu")):
            subprocess.check_call(["make", "-s", "-j8", "-C", HERE, "refcuda", f"REF={REFERENCE_SRC}"],
                                  stdout=subprocess.DEVNULL)


_PROPAGATE_ARGS = [_f64p, C.c_uint32, _u64p, _u8p, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint64,
                   _u64p, _u64p, _u32p, _u32p, C.c_uint32, _u64p, _f64p, _u64p, _u64p, _u8p, C.c_uint32,
                   C.c_int, C.c_double, C.c_double, _f64p]
_LRFU_ARGS = [_f64p, C.c_uint32, _f64p, C.c_uint32, C.c_double, C.c_double, _f64p]

_lib = None
_ref = None
_refcuda = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(REF_DIR, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.kvo_page_mass.argtypes = [
            C.c_void_p, C.c_int, C.c_uint64, C.c_uint64, C.c_uint64,
            C.c_void_p, C.c_int, C.c_uint64, C.c_uint64, C.c_uint64,
            C.c_void_p, C.c_uint64,
            C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
            C.c_uint64, C.c_uint32, C.c_double, C.c_double, C.c_uint32, _f64p]
        L.kvo_recall_fp16.argtypes = [C.c_float, C.POINTER(C.c_float)]
        L.kvo_meank_scores.argtypes = [_f32p, _f32p, _u32p, C.c_uint32, C.c_uint32, C.c_uint32,
                                       C.c_uint32, C.c_uint32, C.c_uint32, _u8p, C.c_int, C.c_double, _f64p]
        L.kvo_query_score_frame.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                            _u32p, C.c_uint32, C.c_uint64, _u64p, _u32p, _u8p, _u8p,
                                            C.POINTER(C.c_uint64)]
        L.kvo_pick_scored.argtypes = [C.c_uint32, _u32p, _f64p, C.c_uint32, _u32p, C.c_uint32, C.c_uint32,
                                      C.c_int, C.c_uint32, _u32p, C.c_uint32, _u32p, C.POINTER(C.c_uint32)]
        L.kvo_plan_residency.argtypes = [_u64p, C.c_uint32, _u64p, C.c_uint32, C.c_int,
                                         _u64p, C.POINTER(C.c_uint32), _u64p, C.POINTER(C.c_uint32),
                                         _u64p, C.POINTER(C.c_uint32)]
        L.kvo_meank_add.argtypes = [_f32p, _u32p, C.c_uint32, C.c_void_p, C.c_int, C.c_uint64, C.c_uint64,
                                    C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint32,
                                    C.c_uint32]
        L.kvo_restore_k.argtypes = [C.c_int, _u8p, _u8p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                    C.c_int32, _f32p, C.c_uint32]
        L.kvo_propagate_scores.argtypes = _PROPAGATE_ARGS
        L.kvo_lrfu_preview.argtypes = _LRFU_ARGS
        L.kvo_decode.argtypes = [C.c_int, C.c_void_p, C.c_uint32]
        L.kvo_decode.restype = C.c_double
        L.kvo_row_bytes.argtypes = [C.c_int, C.c_uint32]
        L.kvo_row_bytes.restype = C.c_uint64
        _lib = L
    return _lib


def ref():
    """The reference's compiled CPU selection library, or None when absent."""
    global _ref
    if _ref is None:
        path = os.path.join(REF_DIR, "libkvref.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.kvref_query_score_frame.argtypes = lib().kvo_query_score_frame.argtypes
        L.kvref_page_softmax_scores.argtypes = [
            _f32p, _u32p, _f32p, _u32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
            C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, _u32p, C.c_uint32, C.c_int,
            C.c_float, _f64p, C.c_uint64]
        L.kvref_recall_fp16.argtypes = [C.c_float, C.POINTER(C.c_float)]
        L.kvref_pick_scored.argtypes = lib().kvo_pick_scored.argtypes
        L.kvref_plan_residency.argtypes = lib().kvo_plan_residency.argtypes
        L.kvref_propagate_scores.argtypes = _PROPAGATE_ARGS
        L.kvref_lrfu_preview.argtypes = _LRFU_ARGS
        L.kvref_layerwise_tile_scores.argtypes = [_u64p, _u32p, _u8p, _u8p, C.c_uint64, C.c_uint64, C.c_uint32,
                                                  C.c_uint32, C.c_int, _f64p, C.c_uint64, _f64p,
                                                  C.POINTER(C.c_uint64)]
        L.kvref_layerwise_max_page_scores.argtypes = [_f64p, C.c_uint64, _f64p]
        _ref = L
    return _ref


def ref_cuda():
    """The reference's compiled GPU scorers, or None when absent."""
    global _refcuda
    if _refcuda is None:
        path = os.path.join(REF_DIR, "libkvref_cuda.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.kvref_attention_score.argtypes = [
            C.c_void_p, C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint64,
            C.c_void_p, C.c_int, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint64,
            C.c_void_p, C.c_int, C.c_uint64, C.c_float, C.c_float, C.c_uint32,
            _u32p, C.c_uint32, _f32p, C.POINTER(C.c_double)]
        L.kvref_page_softmax_cuda.argtypes = [C.c_int] + ref().kvref_page_softmax_scores.argtypes + [
            C.POINTER(C.c_double)]
        L.kvref_cuda_release.argtypes = []
        _pp = C.POINTER(C.c_void_p)
        L.kvref_stagein.argtypes = [C.c_int, C.c_uint32, _pp, _u64p, _pp, np.ctypeslib.ndpointer(np.int64),
                                    np.ctypeslib.ndpointer(np.int32), C.c_int64, C.c_int, C.c_int, C.c_int,
                                    C.c_int, _f32p, C.c_int, C.c_uint32, _pp, _u64p, _pp]
        _refcuda = L
    return _refcuda


def ref_attention_score(q_ptr: int, q_type: int, *, dim: int, q_rows: int, heads: int, q_row_stride: int,
                        q_head_stride: int, k_ptr: int, k_type: int, tokens: int, kv_heads: int,
                        k_token_stride: int, k_head_stride: int, mask_ptr: int, mask_type: int,
                        mask_row_stride: int, scale: float, softcap: float, block: int, rows) -> tuple:
    """The reference's llama_kvmem_attention_cuda::score on device buffers (raw
    pointers of the current CUDA device). Returns (mass [len(rows)][pages] f32,
    host ms of the call). The reference always takes a mask; pass a zero one
    for "no mask". Raises on a rejected or unsupported input."""
    rows = np.ascontiguousarray(rows, np.uint32)
    pages = -(-tokens // block)
    out = np.zeros(len(rows) * pages, np.float32)
    ms = C.c_double()
    rc = ref_cuda().kvref_attention_score(q_ptr, q_type, dim, q_rows, heads, q_row_stride, q_head_stride, k_ptr,
                                          k_type, tokens, kv_heads, k_token_stride, k_head_stride, mask_ptr,
                                          mask_type, mask_row_stride, scale, softcap, block, rows, len(rows), out,
                                          C.byref(ms))
    if rc:
        raise ValueError(f"reference attention score failed (rc={rc})")
    return out.reshape(len(rows), pages), ms.value


def ref_page_softmax_cuda(device, sums, counts, q, layer_rows, *, heads, kv_heads, dim, block, accepted, budget,
                          sink, recent, fixed=(), aggregation=0, scale=0.0) -> tuple:
    """The reference's PageSoftmaxCuda::score on `device` over a RawKvStore built
    from K sums (as ref_page_softmax_scores). Returns (scores [P] f64, host ms)."""
    sums = np.ascontiguousarray(sums, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    L, P, _ = sums.shape
    R = q.shape[1]
    out = np.zeros(P + 1, np.float64)
    fx = np.ascontiguousarray(list(fixed) or [0], np.uint32)
    ms = C.c_double()
    rc = ref_cuda().kvref_page_softmax_cuda(device, sums.reshape(-1), np.ascontiguousarray(counts, np.uint32),
                                            q.reshape(-1), np.ascontiguousarray(layer_rows, np.uint32), L, R,
                                            heads, kv_heads, dim, block, accepted, budget, sink, recent, fx,
                                            len(fixed), aggregation, scale, out, P, C.byref(ms))
    if rc:
        raise ValueError(f"reference PageSoftmaxCuda::score failed (rc={rc})")
    return out[:P], ms.value


def ref_stagein(ktype: int, k_items, *, n_head: int, dim: int, n_rot: int = 0, theta=None, nrot: int = 0,
                v_items=()):
    """The reference's stage-in route (kvmem_stagein_enqueue_k / _v + kvmem_stagein_flush,
    src/adapter/llama-kvmem-stagein.cu) for K items (host bytes, device dst pointer, tokens, pos0)
    with the raw-K restore transform, and V items (host bytes, device dst pointer)."""
    nk, nv = len(k_items), len(v_items)
    keep = [np.ascontiguousarray(x[0], np.uint8) for x in k_items] + [np.ascontiguousarray(x[0], np.uint8)
                                                                       for x in v_items]
    vp = C.c_void_p * max(1, nk)
    ks = vp(*[a.ctypes.data for a in keep[:nk]])
    kd = vp(*[x[1] for x in k_items])
    kb = np.array([a.size for a in keep[:nk]] or [0], np.uint64)
    kt = np.array([x[2] for x in k_items] or [0], np.int64)
    kp = np.array([x[3] for x in k_items] or [0], np.int32)
    wp = C.c_void_p * max(1, nv)
    vs = wp(*[a.ctypes.data for a in keep[nk:]])
    vd = wp(*[x[1] for x in v_items])
    vb = np.array([a.size for a in keep[nk:]] or [0], np.uint64)
    # The route rotates every K item and refuses to run without a device theta table
    # (rope_from_dev, llama-kvmem-stagein.cu:557-569); with n_rot = 0 the table is never read,
    # so a one-element placeholder stands in for the engine's frequencies.
    th = np.ascontiguousarray(list(theta)[: n_rot // 2] if theta is not None and n_rot else [1.0], np.float32)
    rc = ref_cuda().kvref_stagein(ktype, nk, C.cast(ks, C.POINTER(C.c_void_p)), kb, C.cast(kd, C.POINTER(C.c_void_p)),
                                  kt, kp, n_head * dim, nrot, n_head, dim, n_rot, th,
                                  len(th), nv, C.cast(vs, C.POINTER(C.c_void_p)), vb,
                                  C.cast(vd, C.POINTER(C.c_void_p)))
    if rc:
        raise ValueError(f"reference stage-in refused (rc={rc})")


def row_bytes(ktype: int, dim: int) -> int:
    return int(lib().kvo_row_bytes(ktype, dim))


def page_mass(q: np.ndarray, q_type: int, k: np.ndarray, k_type: int, *, layers: int, rows: int,
              heads: int, kv_heads: int, dim: int, tokens: int, page_tokens: int, scale: float,
              softcap: float = 0.0, groups: int = 1, mask: np.ndarray | None = None,
              q_strides=None, k_strides=None) -> np.ndarray:
    """FP64 per-token page mass [layers, groups, rows, pages].

    q: bytes of [layers][rows][heads][dim] elements of q_type (dense unless
    q_strides=(layer, row, head) byte strides are given).
    k: bytes of [layers][tokens_alloc][kv_heads] rows of k_type (dense unless
    k_strides=(layer, token, head) byte strides are given).
    mask: optional f32 [rows][>=tokens] bias.
    """
    esz = {F32: 4, F16: 2, BF16: 2}[q_type]
    if q_strides is None:
        q_strides = (rows * heads * dim * esz, heads * dim * esz, dim * esz)
    rb = row_bytes(k_type, dim)
    pages = -(-tokens // page_tokens)
    if k_strides is None:
        k_strides = (pages * page_tokens * kv_heads * rb, kv_heads * rb, rb)
    qb = np.ascontiguousarray(q).view(np.uint8)
    kb = np.ascontiguousarray(k).view(np.uint8)
    out = np.zeros(layers * groups * rows * pages, np.float64)
    mptr, mrow = None, 0
    if mask is not None:
        mask = np.ascontiguousarray(mask, np.float32)
        mptr, mrow = mask.ctypes.data, mask.shape[1]
    rc = lib().kvo_page_mass(qb.ctypes.data, q_type, *q_strides, kb.ctypes.data, k_type, *k_strides,
                             mptr, mrow, layers, rows, heads, kv_heads, dim, tokens, page_tokens,
                             scale, softcap, groups, out)
    if rc:
        raise ValueError(f"oracle page_mass rejected its geometry (rc={rc})")
    return out.reshape(layers, groups, rows, pages)


def recall_fp16(value: float, use_ref: bool = False) -> float:
    out = C.c_float()
    fn = ref().kvref_recall_fp16 if use_ref else lib().kvo_recall_fp16
    rc = fn(value, C.byref(out))
    if rc:
        raise ValueError("recall operand rejected")
    return out.value


def meank_add(sums: np.ndarray, counts: np.ndarray, k: np.ndarray, k_type: int, *, layers: int, kv_heads: int,
              dim: int, tok0: int, n: int, page_tokens: int, k_strides=None) -> int:
    """In place: sums [L][P][Hkv*dim] f32 += K rows of tokens [tok0, tok0+n) (token order, f32 adds),
    counts [P] u32 += tokens per page. k: bytes [L][T][Hkv][row_bytes] (or k_strides =
    (layer, token, head) in bytes). Returns the oracle's status (0 ok)."""
    assert sums.dtype == np.float32 and sums.flags.c_contiguous and counts.dtype == np.uint32
    rb = row_bytes(k_type, dim)
    ls, ts, hs = k_strides or (k.shape[1] * kv_heads * rb, kv_heads * rb, rb)
    kb = np.ascontiguousarray(k).view(np.uint8)
    return int(lib().kvo_meank_add(sums, counts, sums.shape[1],
                                   kb.ctypes.data, k_type, ls, ts, hs, layers, kv_heads, dim, tok0, n,
                                   page_tokens))


def meank_scores(means: np.ndarray, q: np.ndarray, layer_rows, *, heads: int, kv_heads: int, dim: int,
                 score_mask, aggregation: int = 0, scale: float = 0.0) -> np.ndarray:
    """FP64 Mean-K page softmax. means [L][P][Hkv*D] f32, q [L][R][Hq*D] f32."""
    means = np.ascontiguousarray(means, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    L, P, _ = means.shape
    R = q.shape[1]
    out = np.zeros(P, np.float64)
    rc = lib().kvo_meank_scores(means.reshape(-1), q.reshape(-1), np.ascontiguousarray(layer_rows, np.uint32),
                                L, R, heads, kv_heads, dim, P, np.ascontiguousarray(score_mask, np.uint8),
                                aggregation, scale, out)
    if rc:
        raise ValueError(f"oracle meank rejected its operands (rc={rc})")
    return out


def query_score_frame(accepted, block, budget, sink, recent, fixed=(), use_ref=False):
    n_cap = accepted // block + 2
    starts = np.zeros(n_cap, np.uint64)
    counts = np.zeros(n_cap, np.uint32)
    sm = np.zeros(n_cap, np.uint8)
    tm = np.zeros(n_cap, np.uint8)
    n = C.c_uint64()
    fx = np.ascontiguousarray(list(fixed) or [0], np.uint32)
    fn = ref().kvref_query_score_frame if use_ref else lib().kvo_query_score_frame
    rc = fn(accepted, block, budget, sink, recent, fx, len(fixed), n_cap, starts, counts, sm, tm, C.byref(n))
    if rc:
        raise ValueError(f"query_score_frame rejected (rc={rc})")
    k = n.value
    return dict(starts=starts[:k], counts=counts[:k], score_mask=sm[:k], transport_mask=tm[:k],
                accepted_through=accepted)


def pick_scored(n, candidates, scores, mandatory, budget, signed=False, block_tokens=1, ranges=(),
                use_ref=False):
    """Returns (status, ascending ids or None)."""
    cand = np.ascontiguousarray(candidates, np.uint32)
    sc = np.ascontiguousarray(scores, np.float64)
    mand = np.ascontiguousarray(list(mandatory) or [0], np.uint32)
    rg = np.ascontiguousarray(np.asarray(ranges, np.uint32).reshape(-1) if len(ranges) else [0, 0], np.uint32)
    out = np.zeros(max(n, 1), np.uint32)
    cnt = C.c_uint32()
    fn = ref().kvref_pick_scored if use_ref else lib().kvo_pick_scored
    rc = fn(n, cand if len(cand) else np.zeros(1, np.uint32), sc if len(sc) else np.zeros(1),
            len(cand), mand, len(mandatory), budget, int(signed), block_tokens, rg, len(ranges), out,
            C.byref(cnt))
    return rc, (out[:cnt.value].copy() if rc == 0 else None)


def plan_residency(resident, selected, force_reload=False, use_ref=False):
    a = np.ascontiguousarray(list(resident) or [0], np.uint64)
    b = np.ascontiguousarray(list(selected) or [0], np.uint64)
    na, nb = len(resident), len(selected)
    ev = np.zeros(max(na, 1), np.uint64)
    rt = np.zeros(max(na, 1), np.uint64)
    rs = np.zeros(max(nb, 1), np.uint64)
    ne, nr, ns = C.c_uint32(), C.c_uint32(), C.c_uint32()
    fn = ref().kvref_plan_residency if use_ref else lib().kvo_plan_residency
    rc = fn(a, na, b, nb, int(force_reload), ev, C.byref(ne), rt, C.byref(nr), rs, C.byref(ns))
    if rc:
        return rc, None
    return 0, dict(evict=ev[:ne.value].copy(), retain=rt[:nr.value].copy(), restore=rs[:ns.value].copy())


def ref_page_softmax_scores(sums, counts, q, layer_rows, *, heads, kv_heads, dim, block, accepted, budget,
                            sink, recent, fixed=(), aggregation=0, scale=0.0):
    """The reference's own page_softmax_scores over a RawKvStore built from K sums."""
    sums = np.ascontiguousarray(sums, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    L, P, _ = sums.shape
    R = q.shape[1]
    out = np.zeros(P + 1, np.float64)
    fx = np.ascontiguousarray(list(fixed) or [0], np.uint32)
    rc = ref().kvref_page_softmax_scores(sums.reshape(-1), np.ascontiguousarray(counts, np.uint32),
                                         q.reshape(-1), np.ascontiguousarray(layer_rows, np.uint32), L, R,
                                         heads, kv_heads, dim, block, accepted, budget, sink, recent, fx,
                                         len(fixed), aggregation, scale, out, P)
    if rc:
        raise ValueError(f"reference page_softmax_scores rejected (rc={rc})")
    return out[:P]


def ref_layerwise_tile_scores(frame: dict, page_tokens: int, mean_tokens: int, keep_halves: bool, masses):
    """The reference's layerwise_tile_scores of one tile whose scorer returned `masses`
    (over the half-page frame when mean_tokens = page_tokens / 2). Raises on a rejection."""
    n = len(frame["starts"])
    masses = np.ascontiguousarray(masses, np.float64)
    out = np.zeros(2 * n + 1, np.float64)
    k = C.c_uint64()
    rc = ref().kvref_layerwise_tile_scores(np.ascontiguousarray(frame["starts"], np.uint64),
                                           np.ascontiguousarray(frame["counts"], np.uint32),
                                           np.ascontiguousarray(frame["score_mask"], np.uint8),
                                           np.ascontiguousarray(frame["transport_mask"], np.uint8), n,
                                           frame["accepted_through"], page_tokens, mean_tokens, int(keep_halves),
                                           masses, len(masses), out, C.byref(k))
    if rc:
        raise ValueError(f"reference layerwise_tile_scores rejected (rc={rc})")
    return out[:k.value].copy()


def ref_layerwise_max_page_scores(halves):
    halves = np.ascontiguousarray(halves, np.float64)
    out = np.zeros(max(1, len(halves) // 2), np.float64)
    rc = ref().kvref_layerwise_max_page_scores(halves, len(halves), out)
    if rc:
        raise ValueError(f"reference layerwise_max_page_scores rejected (rc={rc})")
    return out[: len(halves) // 2]


def _graph_arrays(graph):
    """graph: dict(block, accepted, completed, rows=[(source, samples, [(target, mass), ...])],
    spans=None | [(begin, end, end_known)])."""
    rows = graph.get("rows", [])
    src = np.array([r[0] for r in rows] or [0], np.uint64)
    smp = np.array([r[1] for r in rows] or [0], np.uint64)
    cnt = np.array([len(r[2]) for r in rows] or [0], np.uint32)
    beg = np.concatenate([[0], np.cumsum(cnt)[:-1]]).astype(np.uint32) if rows else np.zeros(1, np.uint32)
    edges = [e for r in rows for e in r[2]]
    tgt = np.array([e[0] for e in edges] or [0], np.uint64)
    mass = np.array([e[1] for e in edges] or [0.0], np.float64)
    spans = graph.get("spans")
    sb = np.array([x[0] for x in spans or []] or [0], np.uint64)
    se = np.array([x[1] for x in spans or []] or [0], np.uint64)
    sk = np.array([1 if x[2] else 0 for x in spans or []] or [0], np.uint8)
    return src, smp, beg, cnt, len(rows), tgt, mass, sb, se, sk, len(spans or []), 1 if spans is not None else 0


def propagate_scores(raw, starts, transport_mask, accepted, graph, alpha=0.2, cross=0.25, use_ref=False):
    """(rc, out) of propagate_query_scores: the C restatement, or the reference itself (use_ref)."""
    raw = np.ascontiguousarray(raw, np.float64)
    n = len(raw)
    out = np.zeros(max(1, n), np.float64)
    src, smp, beg, cnt, nrows, tgt, mass, sb, se, sk, ns, hm = _graph_arrays(graph)
    fn = ref().kvref_propagate_scores if use_ref else lib().kvo_propagate_scores
    rc = fn(raw if n else np.zeros(1), n, np.ascontiguousarray(starts, np.uint64),
            np.ascontiguousarray(transport_mask, np.uint8), accepted, graph["block"], graph["accepted"],
            graph["completed"], src, smp, beg, cnt, nrows, tgt, mass, sb, se, sk, ns, hm, alpha, cross, out)
    return int(rc), out[:n]


def lrfu_preview(scores, prev, lam=0.5, fraction=0.9, use_ref=False):
    scores = np.ascontiguousarray(scores, np.float64)
    n_prev = len(prev)
    prev = np.ascontiguousarray(prev if n_prev else [0.0], np.float64)
    n = len(scores)
    out = np.zeros(max(1, n), np.float64)
    fn = ref().kvref_lrfu_preview if use_ref else lib().kvo_lrfu_preview
    rc = fn(scores if n else np.zeros(1), n, prev, n_prev, lam, fraction, out)
    return int(rc), out[:n]


def restore_k(ktype: int, src: np.ndarray, *, tokens: int, n_head: int, dim: int, n_rot: int = 0, pos0: int = 0,
              theta=None, nrot: int = 0):
    """Raw-K restore transform of `tokens` packed rows -> (rc, packed output bytes)."""
    src = np.ascontiguousarray(src, np.uint8).reshape(-1)
    dst = np.zeros_like(src)
    # The route rotates every K item and refuses to run without a device theta table
    # (rope_from_dev, llama-kvmem-stagein.cu:557-569); with n_rot = 0 the table is never read,
    # so a one-element placeholder stands in for the engine's frequencies.
    th = np.ascontiguousarray(list(theta)[: n_rot // 2] if theta is not None and n_rot else [1.0], np.float32)
    rc = lib().kvo_restore_k(ktype, src, dst, tokens, n_head, dim, n_rot, pos0, th, nrot)
    return int(rc), dst


def prefill_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, base: int, rows, sample_rows=(),
                      page_tokens: int = 64, pages: int = 0, scale: float = 0.0):
    """FP64 restatement of causal prompt attention with page-LSE capture (the engine's
    causal_softmax_attention_with_page_lse; capture semantics of PromptPageLseRows,
    backends/patches/ninfer-prefill-page-lse-kv-coverage.patch:953-984: per sampled row and
    query head, page LSE = max + log(sum of exp over the page's visible keys); pages with no
    visible key stay at the -inf of clear_prompt_page_lse, :925-928 and :945-947).

    q [width][Hq][D], k / v [T][Hkv][D] (any float dtype, read as float64); prompt row i sits at
    position base + i and sees keys 0 .. base + i. Returns (out [len(rows)][Hq][D] for the listed
    rows, lse [len(sample_rows)][Hq][pages] natural log)."""
    width, hq, dim = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    sc = scale if scale > 0 else 1.0 / np.sqrt(dim)
    pages = pages or -(-(base + width) // page_tokens)

    def logits(r):
        n = base + r + 1
        qr = q[r].astype(np.float64)                                   # [Hq][D]
        kk = k[:n].astype(np.float64)                                  # [n][Hkv][D]
        kq = np.repeat(kk, g, axis=1)                                  # [n][Hq][D]
        return sc * np.einsum("hd,nhd->hn", qr, kq), n                 # [Hq][n]

    out = np.zeros((len(rows), hq, dim), np.float64)
    for i, r in enumerate(rows):
        s, n = logits(r)
        m = s.max(axis=1, keepdims=True)
        p = np.exp(s - m)
        vv = np.repeat(v[:n].astype(np.float64), g, axis=1)            # [n][Hq][D]
        out[i] = np.einsum("hn,nhd->hd", p, vv) / p.sum(axis=1)[:, None]
    lse = np.full((len(sample_rows), hq, pages), -np.inf, np.float64)
    for i, r in enumerate(sample_rows):
        s, n = logits(r)
        npg = -(-n // page_tokens)
        padded = np.full((hq, npg * page_tokens), -np.inf)
        padded[:, :n] = s
        blk = padded.reshape(hq, npg, page_tokens)                     # every page has a visible key
        m = blk.max(axis=2)
        lse[i, :, :npg] = m + np.log(np.exp(blk - m[..., None]).sum(axis=2))
    return out, lse


def page_mass_from_lse(lse: np.ndarray) -> np.ndarray:
    """FP64 page mass of captured prefill LSE [samples][Hq][pages]: softmax over the pages of
    each (sample, head), then the mean over heads (attention_page_mass_from_lse,
    ninfer-prefill-page-lse-kv-coverage.patch:6-7, "exactly as in the independent
    attention_page_mass path": the normalize / average kernels of
    src/adapter/llama-kvmem-attention-cuda.cu:98-121). Returns [samples][pages]."""
    m = lse.max(axis=2, keepdims=True)
    e = np.where(np.isfinite(lse), np.exp(lse - m), 0.0)
    return (e / e.sum(axis=2, keepdims=True)).mean(axis=1)
