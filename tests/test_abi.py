"""CPU tests: the C-ABI library loads and exports every function include/kvm_recall.h declares."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^\s*(?:int|size_t|uint64_t|const\s+uint8_t\s*\*)\s*(kvm_\w+)\s*\(", src, flags=re.M)
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("kvm_score_pages", "kvm_select_topk", "kvm_plan_residency", "kvm_stagein_pool", "kvm_meank_score",
              "kvm_recall_step"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import kvmem_b200._abi as A
    lib = A.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # every binding signature names a declared function
    assert set(A.SIGNATURES) == set(declared_functions())


def test_row_bytes_host_only():
    import kvmem_b200 as K
    assert K.row_bytes(K.F16, 256) == 512
    assert K.row_bytes(K.Q8_0, 256) == 272
    assert K.row_bytes(K.Q4_0, 256) == 144
    assert K.row_bytes(K.Q5_0, 128) == 88
    assert K._abi.load().kvm_row_bytes(99, 128) == 0


def test_context_without_gpu_reports_cuda_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import kvmem_b200 as K
    with pytest.raises(K.KvmError) as e:
        K.RecallContext(0)
    assert e.value.code == K._abi.ERR_CUDA
