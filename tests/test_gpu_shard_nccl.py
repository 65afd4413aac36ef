"""Sharded selection and recall across 2 GPUs with NCCL all-gathers (skipped with fewer GPUs).

Runs tests/shard_nccl_worker.py under torchrun (one rank per GPU, 127.0.0.1
rendezvous, bounded by a timeout) and checks that every rank ends with the same
selection as the unsharded top-k of the whole history (with either exchange:
statistics + candidates, or one all-gather of the page LSE), and that the sharded
recall step (kvmem_b200.shard.ShardedRecall) leaves rank 0's paged cache holding
exactly the host records of the selected pages, each rank having written the
pages of its own range (rank 1 through a CUDA-IPC peer mapping).
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_nccl_sharded_selection(tmp_path):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(HERE, "shard_nccl_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    if r.returncode != 0:
        lines = [x for x in (r.stdout + r.stderr).splitlines() if "rank" in x or "Error" in x or "error" in x]
        raise AssertionError("torchrun workers failed:\n" + "\n".join(lines[:80]))
    res = [json.load(open(tmp_path / f"rank{i}.json")) for i in range(2)]
    assert res[0]["status"] == 0 and res[1]["status"] == 0
    assert res[0]["ids"] == res[1]["ids"] == res[0]["unsharded"]
    assert res[0]["ids_lse"] == res[1]["ids_lse"] == res[0]["unsharded"]
    # sharded recall (both exchanges): each rank's restored pages written into rank 0's cache over NVLink
    for key in ("recall", "recall_lse"):
        for r in res:
            assert r[key]["steps"] == 3 and r[key]["status"] == 0
        assert res[0][key]["bad"] == [], res[0][key]["bad"][:10]
