"""GPU: the reference's own interfaces, implemented over the C ABI by the adapters in
kvmem_b200/adapter, driven by a C++ test compiled against the reference's headers
(tests/cpp/adapters_test.cpp):

* llama_kvmem_attention_cuda::score (src/adapter/llama-kvmem-attention-cuda.h:9-18):
  sampled rows in one call, a device and a host (staged) mask, against the FP64
  restatement within 1e-3 relative; false outside the kernel's domain;
* kvmem::PageSoftmaxCuda (kvmem/include/kvmem/page_softmax_cuda.hpp:10-31): score
  with its own and with a borrowed workspace, score_current_layer on native FP16
  queries, Mean and Max aggregation, against the reference's own page_softmax_scores
  within its qualification bound; std::invalid_argument for a non-finite operand and
  a too-small workspace.

The binary is built by ``make -C tests/cpp`` (``__graft_entry__.build()``) where the
reference headers are available, and travels with the tree."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cpp", "_build", "adapters_test")


def test_reference_interfaces_over_the_b200_library():
    assert os.path.exists(BIN), "tests/cpp/_build/adapters_test is not built (make -C tests/cpp)"
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok")
