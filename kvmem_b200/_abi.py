"""ctypes binding of the C ABI declared in ``include/kvm_recall.h``.

The shared library ``kvmem_b200/_lib/libkvm_b200.so`` is built in-tree by
``kvmem_b200/build.py``. There is no fallback: if the library is missing and
cannot be built, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os
import shutil

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libkvm_b200.so")

# kvm_status
OK = 0
ERR_INVALID_PLAN = 1
ERR_UNSUPPORTED = 2
ERR_BUDGET_EXCEEDED = 3
ERR_STALE = 4
ERR_PENDING = 5
ERR_TRANSFER_FAILED = 6
ERR_DISCONNECTED = 7
ERR_INVALID_SESSION = 8
ERR_INVALID_ARGUMENT = 9
ERR_LENGTH = 10
ERR_CUDA = 11
ERR_TIMEOUT = 12
ERR_NONFINITE = 13
STATUS_NAMES = {
    0: "KVM_OK", 1: "KVM_ERR_INVALID_PLAN", 2: "KVM_ERR_UNSUPPORTED", 3: "KVM_ERR_BUDGET_EXCEEDED",
    4: "KVM_ERR_STALE", 5: "KVM_ERR_PENDING", 6: "KVM_ERR_TRANSFER_FAILED", 7: "KVM_ERR_DISCONNECTED",
    8: "KVM_ERR_INVALID_SESSION", 9: "KVM_ERR_INVALID_ARGUMENT", 10: "KVM_ERR_LENGTH", 11: "KVM_ERR_CUDA",
    12: "KVM_ERR_TIMEOUT", 13: "KVM_ERR_NONFINITE",
}

# kvm_type
F32, F16, BF16, Q8_0, Q4_0, Q5_0 = 0, 1, 2, 3, 4, 5

IPC_HANDLE_BYTES = 72  # KVM_IPC_HANDLE_BYTES


class KvmError(RuntimeError):
    """A non-zero kvm_status. ``code`` is the status value."""

    def __init__(self, code: int, where: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(code, code)}")
        self.code = code


class Query(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("rows", C.c_uint32),
                ("layer_stride", C.c_uint64), ("row_stride", C.c_uint64), ("head_stride", C.c_uint64),
                ("row_ids", C.POINTER(C.c_uint32)), ("row_count", C.c_uint32), ("reserved", C.c_uint32)]


class KCache(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("reserved", C.c_uint32),
                ("layer_stride", C.c_uint64), ("token_stride", C.c_uint64), ("head_stride", C.c_uint64),
                ("capacity_tokens", C.c_uint64)]


class ScoreDesc(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("q_heads", C.c_uint32), ("kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("tokens", C.c_uint64), ("page_tokens", C.c_uint32),
                ("groups", C.c_uint32), ("scale", C.c_float), ("softcap", C.c_float), ("mask", C.c_void_p),
                ("mask_type", C.c_int32), ("reserved", C.c_uint32), ("mask_row_stride", C.c_uint64)]


class StageLayout(C.Structure):
    _fields_ = [("planes", C.c_uint32), ("reserved", C.c_uint32),
                ("host_base", C.c_void_p * 2), ("host_row_stride", C.c_uint64 * 2),
                ("host_page_stride", C.c_uint64 * 2), ("dev_base", C.c_void_p * 2),
                ("dev_row_stride", C.c_uint64 * 2), ("dev_slot_stride", C.c_uint64 * 2),
                ("bytes", C.c_uint64 * 2)]


class Copy(C.Structure):
    _fields_ = [("src", C.c_void_p), ("dst", C.c_void_p), ("bytes", C.c_uint64)]


class StepDesc(C.Structure):
    _fields_ = [("score", C.POINTER(ScoreDesc)), ("q", C.POINTER(Query)), ("k", C.POINTER(KCache)),
                ("keep", C.POINTER(C.c_uint32)), ("nkeep", C.c_uint32), ("budget", C.c_uint32),
                ("chunks", C.c_uint32), ("stage_ctas", C.c_uint32), ("force_reload", C.c_int),
                ("first_layers", C.c_uint32)]


_vp, _u32, _u64, _i = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int
class RestoreItem(C.Structure):
    _fields_ = [("src", C.c_void_p), ("dst", C.c_void_p), ("tokens", C.c_uint32), ("pos0", C.c_int32)]


class GraphRow(C.Structure):
    _fields_ = [("source", C.c_uint64), ("samples", C.c_uint64), ("edge_begin", C.c_uint32),
                ("edge_count", C.c_uint32)]


class GraphEdge(C.Structure):
    _fields_ = [("target", C.c_uint64), ("mass", C.c_double)]


class GraphSpan(C.Structure):
    _fields_ = [("begin", C.c_uint64), ("end", C.c_uint64), ("end_known", C.c_uint32), ("reserved", C.c_uint32)]


class Graph(C.Structure):
    _fields_ = [("block_tokens", C.c_uint32), ("has_messages", C.c_int32), ("accepted_through", C.c_uint64),
                ("completed_through", C.c_uint64), ("rows", C.POINTER(GraphRow)), ("nrows", C.c_uint32),
                ("nedges", C.c_uint32), ("edges", C.POINTER(GraphEdge)), ("spans", C.POINTER(GraphSpan)),
                ("nspans", C.c_uint32), ("reserved", C.c_uint32)]


class PrefillDesc(C.Structure):
    _fields_ = [("q_heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("type", C.c_int32),
                ("base", C.c_uint64), ("width", C.c_uint32), ("scale", C.c_float), ("page_tokens", C.c_uint32),
                ("pages", C.c_uint32), ("samples", C.c_uint32), ("reserved", C.c_uint32),
                ("sample_rows", C.POINTER(C.c_uint32))]


PREFILL_MAX_SAMPLES = 4096

SIGNATURES = {
    "kvm_ctx_create": ([_i, C.POINTER(C.c_void_p)], _i),
    "kvm_ctx_destroy": ([_vp], _i),
    "kvm_ctx_device": ([_vp], _i),
    "kvm_ctx_status": ([_vp, _vp], _i),
    "kvm_score_workspace_bytes": ([C.POINTER(ScoreDesc), _u32], C.c_size_t),
    "kvm_ctx_bind_workspace": ([_vp, _vp, C.c_size_t], _i),
    "kvm_ctx_device_bytes": ([_vp], C.c_size_t),
    "kvm_score_pages": ([_vp, C.POINTER(ScoreDesc), C.POINTER(Query), C.POINTER(KCache), _vp, _vp, _vp], _i),
    "kvm_score_pages_noalloc": ([C.POINTER(ScoreDesc), C.POINTER(Query), C.POINTER(KCache), _vp, _vp, _vp], _i),
    "kvm_query_fixed_blocks": ([C.c_uint64, _u32, _u32, _u32, _u32, C.POINTER(C.c_uint32), _u32,
                                C.POINTER(C.c_uint32), _u32, C.POINTER(C.c_uint32), _u32, C.POINTER(C.c_uint32)], _i),
    "kvm_query_score_frame": ([C.c_uint64, _u32, _u32, _u32, _u32, C.POINTER(C.c_uint32), _u32, C.c_uint64, _vp,
                               _vp, _vp, _vp, C.POINTER(C.c_uint64)], _i),
    "kvm_select_topk": ([_vp, _vp, _u32, _u32, _u32, C.POINTER(C.c_uint32), _u32, _u32, _i, _vp, _vp, _u32, _vp],
                        _i),
    "kvm_select_topk_media": ([_vp, _vp, _u32, _u32, _u32, C.POINTER(C.c_uint32), _u32, _u32, _i, _u32,
                               C.POINTER(C.c_uint32), _u32, _vp, _vp, _u32, _vp], _i),
    "kvm_pool_create": ([_vp, _u32, _u32, _u32, C.POINTER(C.c_void_p)], _i),
    "kvm_pool_destroy": ([_vp], _i),
    "kvm_pool_reset": ([_vp, _vp], _i),
    "kvm_plan_residency": ([_vp, _vp, _vp, _vp, _u32, _i, _vp, _vp, _vp], _i),
    "kvm_stagein_pool": ([_vp, _vp, C.POINTER(StageLayout), _u32, _vp], _i),
    "kvm_stagein_copies": ([_vp, C.POINTER(Copy), _u32, _u32, _vp], _i),
    "kvm_stagein_wait": ([_vp, _vp, _u64], _i),
    "kvm_stageout_create": ([_i, _u64, _u32, C.POINTER(C.c_void_p)], _i),
    "kvm_stageout_destroy": ([_vp], _i),
    "kvm_stageout_enqueue": ([_vp, _vp, _u64, C.POINTER(C.c_uint64)], _i),
    "kvm_stageout_used": ([_vp], _u64),
    "kvm_stageout_submit": ([_vp, _u32, _vp, C.POINTER(C.c_int)], _i),
    "kvm_stageout_wait": ([_vp, _i, _u64], _i),
    "kvm_stageout_slot_base": ([_vp, _i], _vp),
    "kvm_stageout_clear": ([_vp], _i),
    "kvm_pool_read": ([_vp, _vp, _vp, _vp], _i),
    "kvm_transfer_prepare": ([_vp, _vp, _vp, _vp, _u32, _i, _vp, C.POINTER(C.c_void_p)], _i),
    "kvm_transfer_start_spill": ([_vp, C.POINTER(StageLayout), _vp, _u32, _vp], _i),
    "kvm_transfer_poll": ([_vp], _i),
    "kvm_transfer_start_restore": ([_vp, C.POINTER(StageLayout), _u32, _vp], _i),
    "kvm_transfer_publish": ([_vp, _vp], _i),
    "kvm_transfer_abort": ([_vp, _u64, C.POINTER(C.c_int)], _i),
    "kvm_transfer_destroy": ([_vp], _i),
    "kvm_restore_k": ([_vp, _i, C.POINTER(RestoreItem), _u32, _u32, _u32, _u32, C.POINTER(C.c_float), _u32, _vp],
                      _i),
    "kvm_propagate_scores": ([_vp, _vp, _u32, _vp, _vp, _u64, C.POINTER(Graph), C.c_double, C.c_double, _vp, _vp],
                             _i),
    "kvm_lrfu_preview": ([_vp, _vp, _u32, _vp, _u32, C.c_double, C.c_double, _vp, _vp], _i),
    "kvm_meank_add": ([_vp, C.POINTER(KCache), _u32, _u32, _u32, _u64, _u32, _u32, _vp, _u32, _vp, _vp], _i),
    "kvm_meank_score": ([_vp, _vp, _vp, _vp, C.POINTER(C.c_uint32), _u32, _u32, _u32, _u32, _u32, _u32,
                         C.POINTER(C.c_uint8), _i, C.c_float, _vp, _vp], _i),
    "kvm_layerwise_accumulate": ([_vp, _vp, _u32, _u32, _i, _vp, _vp, _vp], _i),
    "kvm_layerwise_finish": ([_vp, _vp, _u32, _i, _vp, _vp], _i),
    "kvm_recall_step": ([_vp, C.POINTER(StepDesc), _vp, C.POINTER(StageLayout), _vp, _vp, _vp, _vp], _i),
    "kvm_shard_page_lse": ([_vp, C.POINTER(ScoreDesc), C.POINTER(Query), C.POINTER(KCache), _u32, _u32, _vp, _vp],
                           _i),
    "kvm_page_mass_from_lse": ([_vp, C.POINTER(ScoreDesc), _u32, _vp, _vp, _vp, _vp], _i),
    "kvm_shard_score_partial": ([_vp, C.POINTER(ScoreDesc), C.POINTER(Query), C.POINTER(KCache), _u32, _u32, _vp,
                                 _vp], _i),
    "kvm_shard_merge_stats": ([_vp, _vp, _u32, _u32, _vp, _vp], _i),
    "kvm_shard_score_finish": ([_vp, C.POINTER(ScoreDesc), _u32, _u32, _vp, _vp, _vp, _vp], _i),
    "kvm_shard_candidates": ([_vp, _vp, _u32, _u32, _u32, _u32, C.POINTER(C.c_uint32), _u32, _u32, _vp, _vp, _vp],
                             _i),
    "kvm_shard_merge": ([_vp, _vp, _vp, _u32, _u32, _u32, C.POINTER(C.c_uint32), _u32, _u32, _vp, _vp, _u32, _vp],
                        _i),
    "kvm_shard_stagein": ([_vp, _vp, C.POINTER(StageLayout), _u32, _u32, _u32, _vp], _i),
    "kvm_ipc_export": ([_vp, _vp], _i),
    "kvm_ipc_open": ([_i, _vp, C.POINTER(C.c_void_p)], _i),
    "kvm_ipc_close": ([_i, _vp], _i),
    "kvm_prefill_attention": ([_vp, C.POINTER(PrefillDesc), _vp, _u64, _u64, C.POINTER(KCache), C.POINTER(KCache),
                               _vp, _u64, _u64, _vp, _vp], _i),
    "kvm_row_bytes": ([_i, _u32], _u64),
    "kvm_ctx_launches": ([_vp], _u64),
}

_lib = None


def load() -> C.CDLL:
    """Load (building first if absent and nvcc is available) the CUDA library."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
            from . import build as _build
            _build.build()
        else:
            raise RuntimeError(f"kvmem_b200: CUDA library {LIB_PATH} is missing and nvcc is unavailable")
    L = C.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def check(code: int, where: str) -> None:
    if code != OK:
        raise KvmError(code, where)
