"""GPU (two devices): kvm_adapter::ShardedRecallStep, the C++ host side of the page-range
sharded recall step over the C ABI and NCCL (kvmem_b200/adapter/kvm_sharded_step.hpp),
driven by tests/cpp/sharded_step_test.cpp in one process with one thread per device:

* over three steps of a 4-layer, 40-page fp16 history split 20 / 20 (layer chunks 1 + 3),
  both ranks hold exactly the selection kvm_score_pages + kvm_select_topk give over the
  whole history on one device;
* device 0's paged cache holds, in the slots its pools assign, the host records (K and
  V planes) of every selected page, byte for byte: device 1 wrote its range's pages
  through peer access.

The binary is built by ``make -C tests/cpp`` (``__graft_entry__.build()``) and travels
with the tree; it exits 77 (skip) with fewer than two devices."""
import os
import subprocess

import pytest
import torch

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cpp", "_build", "sharded_step_test")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two devices")
def test_sharded_step_adapter_on_two_devices():
    assert os.path.exists(BIN), "tests/cpp/_build/sharded_step_test is not built (make -C tests/cpp)"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300, env=env)
    if r.returncode == 77:
        pytest.skip(r.stdout.strip())
    assert r.returncode == 0, r.stdout + r.stderr
    assert "sharded step ok" in r.stdout
