"""GPU: the reference's own kvmem::MemorySession (kvmem/src/host/memory_contract.cpp:245-365)
drives the C++ memory-backend adapter (kvmem_b200/adapter/kvm_memory_backend.cpp) over the
kvm_transfer_* C ABI: restores, spills of device-written blocks, both abort outcomes, stale
and pending plans, and a backend refusal with the strong guarantee (tests/cpp/memory_session_test.cpp).
The binary is built by ``make -C tests/cpp`` (``__graft_entry__.build()``) where the reference
headers are available and travels with the tree."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cpp", "_build", "memory_session_test")


def test_reference_memory_session_drives_the_b200_backend():
    assert os.path.exists(BIN), "tests/cpp/_build/memory_session_test is not built (make -C tests/cpp)"
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "memory_session_test: OK" in r.stdout
