"""Sharded selection on gloo ranks (CPU): the page partition with either exchange
(ShardedSelector: statistics and candidate all-gathers; LseGatherSelector: one
all-gather of the page LSE, ranges of unequal size padded) gives every rank the
unsharded top-k."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def problem(seed=0):
    rng = np.random.default_rng(seed)
    L, R, Hq, Hkv, D, B, P = 2, 1, 4, 2, 16, 8, 23
    T = P * B - 3
    q = rng.standard_normal((L, R, Hq, D))
    k = rng.standard_normal((L, P * B, Hkv, D))
    k[:, 5 * B:6 * B] += 0.9 * q[:, 0, ::2][:, None, :, :]  # a needle page
    return q, k, T, B, P


def worker(rank, world, port, out_q, kind):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kvmem_b200.shard import LseGatherSelector, ShardGeometry, ShardedSelector, page_ranges
        from tests.shard_cpu import CpuShardCompute
        q, k, T, B, P = problem()
        L, R, Hq = q.shape[0], q.shape[1], q.shape[2]
        p0, p1 = page_ranges(P, world)[rank]
        geo = ShardGeometry(layers=L, rows=R, q_heads=Hq, kv_heads=k.shape[2], groups=1, total_pages=P, page0=p0,
                            local_pages=p1 - p0)
        cls = LseGatherSelector if kind == "lse" else ShardedSelector
        sel = cls(CpuShardCompute(q, k, T, B, 0.25))
        ids, n = sel.select(None, None, None, geo, keep=[0, P - 1], budget=6)
        out_q.put((rank, ids.numpy().tolist(), n.numpy().tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,kind", [(2, "candidates"), (3, "candidates"), (2, "lse"), (3, "lse")])
def test_sharded_selection_equals_unsharded(world, kind):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, out_q, kind)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out_q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, T, B, P = problem()
    L = q.shape[0]
    # Unsharded: FP64 oracle page mass of the whole history, then pick_scored_blocks.
    qb = q.astype(np.float32)
    kb = k.astype(np.float32)
    mass = O.page_mass(qb, O.F32, kb, O.F32, layers=L, rows=1, heads=q.shape[2], kv_heads=k.shape[2],
                       dim=q.shape[3], tokens=T, page_tokens=B, scale=0.25)[:, 0, 0]
    want = []
    for l in range(L):
        rc, ids = O.pick_scored(P, list(range(P)), mass[l], [0, P - 1], 6)
        want.append(ids.tolist())
    for rank, ids, n in results:
        got = [ids[l][: n[l]] for l in range(L)]
        assert got == want, (rank, got, want)
