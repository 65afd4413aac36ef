"""CPU: the C++ adapters (kvmem_b200/adapter: the memory backend, llama_kvmem_attention_cuda,
kvmem::PageSoftmaxCuda, the page-range sharded recall step) and their tests compile against the reference's own headers and link
against libkvm_b200.so and the reference build (runs where the reference headers and the
libraries are present)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("KVM_REFERENCE_SRC") or os.path.normpath(os.path.join(ROOT, os.pardir, "reference"))


def test_adapter_compiles_against_the_reference_contract(tmp_path):
    need = [os.path.join(REF, "kvmem", "include", "kvmem", "memory_contract.hpp"),
            os.path.join(ROOT, "oracle", "_ref", "libkvref.so"),
            os.path.join(ROOT, "kvmem_b200", "_lib", "libkvm_b200.so")]
    missing = [p for p in need if not os.path.exists(p)]
    if missing:
        pytest.skip(f"not available here: {missing}")
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), f"REF={REF}", f"OUT={tmp_path}"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert os.path.exists(os.path.join(tmp_path, "memory_session_test"))
    assert os.path.exists(os.path.join(tmp_path, "adapters_test"))
    assert os.path.exists(os.path.join(tmp_path, "sharded_step_test"))
