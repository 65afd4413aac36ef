"""kvmem_b200 — B200-native history recall for KVMem.

Scores every page of a paged KV history against the current queries
(page-softmax mass under GQA), selects the top-k pages with pinned keep pages,
plans the residency delta and stages the selected pages from mapped pinned
host memory into a device paged cache. The compute lives in the CUDA library
``_lib/libkvm_b200.so`` (C ABI: ``include/kvm_recall.h``); this package is the
host-side binding.
"""
from . import _abi
from ._abi import KvmError, F32, F16, BF16, Q8_0, Q4_0, Q5_0
from .recall import (AttentionCuda, PageSoftmaxCuda, RecallContext, ResidencyPool, StageOut, TensorView, Transfer,
                     ipc_close, ipc_export, ipc_open, pick_scored_blocks, row_bytes, stage_layout)

__all__ = ["KvmError", "F32", "F16", "BF16", "Q8_0", "Q4_0", "Q5_0", "AttentionCuda", "PageSoftmaxCuda",
           "RecallContext", "ResidencyPool", "StageOut", "TensorView", "Transfer", "ipc_close", "ipc_export",
           "ipc_open", "pick_scored_blocks", "row_bytes", "stage_layout"]
