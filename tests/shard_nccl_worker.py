"""torchrun worker for tests/test_gpu_shard_nccl.py: one rank per GPU, NCCL all-gathers.

Every rank generates the same seeded problem, keeps its page range's K on its
GPU, runs the sharded selection and writes its selection to <out>/rank<r>.json;
rank 0 also writes the unsharded selection of the whole history on its GPU.
"""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(out_dir):
    import kvmem_b200 as K
    from kvmem_b200.shard import ShardCompute, ShardedSelector, ShardGeometry, page_ranges
    from tests import util as U
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    try:
        rng = np.random.default_rng(7)
        L, Hq, Hkv, D, B, P = 3, 24, 4, 256, 64, 50
        T = P * B - 5
        qb = U.make_q(rng, U.F32, L, 1, Hq, D)
        qdir = qb.view(np.float32).reshape(L, 1, Hq, D)[:, 0].reshape(L, Hkv, Hq // Hkv, D).mean(axis=2)
        qdir /= np.sqrt((qdir ** 2).mean(axis=-1, keepdims=True))
        needles = (2, 9, 13, 21, 30, 38, 41, 47)  # 8 needles + 2 keep pages = the budget: a wide boundary gap
        kb = U.make_k(rng, U.F16, L, P * B, Hkv, D, needle_pages=needles, page=B, q_dir=qdir / np.sqrt(D))
        dev = torch.device("cuda", local)
        p0, p1 = page_ranges(P, world)[rank]
        k_local = torch.from_numpy(np.ascontiguousarray(kb[:, p0 * B:p1 * B]).reshape(-1)).to(dev)
        q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, 1, Hq, D)
        desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=B)
        q = K.RecallContext.make_query(q_d, 1)
        kc = K.RecallContext.make_kcache(k_local, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=(p1 - p0) * B)
        ctx = K.RecallContext(local)
        geo = ShardGeometry(layers=L, rows=1, q_heads=Hq, kv_heads=Hkv, groups=1, total_pages=P, page0=p0,
                            local_pages=p1 - p0)
        ids, n = ShardedSelector(ShardCompute(ctx)).select(desc, q, kc, geo, keep=[0, P - 1], budget=10)
        torch.cuda.synchronize()
        res = {"ids": [ids[l, : int(n[l])].tolist() for l in range(L)], "status": ctx.status()}
        if rank == 0:
            k_full = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
            full = K.RecallContext.make_kcache(k_full, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=P * B)
            _, mass = ctx.score_pages(desc, q, full, want_rows=False)
            rid, rn = ctx.select_topk(mass.view(L, P), [0, P - 1], 10)
            res["unsharded"] = [rid[l, : int(rn[l])].tolist() for l in range(L)]
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
