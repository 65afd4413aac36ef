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


def sharded_recall_check(K, ctx, kb, qb, rank, world, local, dev, L, Hq, Hkv, D, B, P, T, lse_gather=False):
    """ShardedRecall over 3 steps with changing queries: every rank gathers the restores of its
    page range from its own records into rank 0's cache (a CUDA-IPC peer mapping on rank 1);
    rank 0 then checks every resident slot against the full host records, byte for byte."""
    from kvmem_b200.shard import (LseGatherSelector, ShardCompute, ShardedRecall, ShardedSelector, ShardGeometry,
                                  page_ranges)
    from tests import util as U
    p0, p1 = page_ranges(P, world)[rank]
    lp = p1 - p0
    rb = U.row_bytes(U.F16, D)
    page_k = B * Hkv * rb
    page_v = 160  # V records: 160 bytes per page
    rng = np.random.default_rng(11)
    v_full = rng.integers(0, 256, (L, P, page_v), dtype=np.uint8)
    k_full = kb.reshape(L, P, page_k)
    host_k = torch.from_numpy(np.ascontiguousarray(k_full[:, p0:p1]).reshape(-1)).pin_memory()
    host_v = torch.from_numpy(np.ascontiguousarray(v_full[:, p0:p1]).reshape(-1)).pin_memory()
    slots, budget = 10, 10
    if rank == 0:
        cache_k = torch.zeros(L * slots * page_k, dtype=torch.uint8, device=dev)
        cache_v = torch.zeros(L * slots * page_v, dtype=torch.uint8, device=dev)
        box = [[K.ipc_export(cache_k), K.ipc_export(cache_v)]]
    else:
        box = [None]
    dist.broadcast_object_list(box, src=0)
    ck, cv = (cache_k.data_ptr(), cache_v.data_ptr()) if rank == 0 else (K.ipc_open(local, box[0][0]),
                                                                         K.ipc_open(local, box[0][1]))
    chunk_layers = [(0, 2), (2, L - 2)]
    pools, layouts = [], []
    for l0, nl in chunk_layers:
        pools.append(K.ResidencyPool(ctx, nl, P, slots))
        layouts.append(K.stage_layout([
            dict(host_base=host_k.data_ptr() + l0 * lp * page_k, host_row_stride=lp * page_k,
                 host_page_stride=page_k, dev_base=ck + l0 * slots * page_k, dev_row_stride=slots * page_k,
                 dev_slot_stride=page_k, bytes=page_k),
            dict(host_base=host_v.data_ptr() + l0 * lp * page_v, host_row_stride=lp * page_v,
                 host_page_stride=page_v, dev_base=cv + l0 * slots * page_v, dev_row_stride=slots * page_v,
                 dev_slot_stride=page_v, bytes=page_v)]))
    geo = ShardGeometry(layers=L, rows=1, q_heads=Hq, kv_heads=Hkv, groups=1, total_pages=P, page0=p0,
                        local_pages=lp)
    cls = LseGatherSelector if lse_gather else ShardedSelector
    rec = ShardedRecall(cls(ShardCompute(ctx)), pools, layouts, chunk_layers, geo, stage_ctas=4)
    k_local = torch.from_numpy(np.ascontiguousarray(kb[:, p0 * B:p1 * B]).reshape(-1)).to(dev)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=B)
    kc = K.RecallContext.make_kcache(k_local, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=lp * B)
    qrng = np.random.default_rng(5)
    out = {"steps": 0, "bad": []}
    for step in range(3):
        qs = qb if step == 0 else U.make_q(qrng, U.F32, L, 1, Hq, D)
        q_d = torch.from_numpy(qs.reshape(-1).copy()).to(dev).view(torch.float32).view(L, 1, Hq, D)
        ids, n = rec.step(desc, q_d, kc, [0, P - 1], budget)
        torch.cuda.synchronize()
        if rank == 0:
            ih, nh = ids.cpu().numpy(), n.cpu().numpy()
            ckh = cache_k.cpu().numpy().reshape(L, slots, page_k)
            cvh = cache_v.cpu().numpy().reshape(L, slots, page_v)
            for ci, (l0, nl) in enumerate(chunk_layers):
                slot_of, _ = pools[ci].read()
                for r in range(nl):
                    l = l0 + r
                    sel = ih[l, : nh[l]].tolist()
                    if sorted(np.nonzero(slot_of[r] >= 0)[0].tolist()) != sel:
                        out["bad"].append(f"step {step} layer {l}: residency != selection")
                    for p in sel:
                        s_ = int(slot_of[r, p])
                        if not (np.array_equal(ckh[l, s_], k_full[l, p]) and np.array_equal(cvh[l, s_], v_full[l, p])):
                            out["bad"].append(f"step {step} layer {l} page {p}: bytes differ")
        out["steps"] += 1
    for p in pools:
        p.close()
    dist.barrier()
    if rank != 0:
        K.ipc_close(local, ck)
        K.ipc_close(local, cv)
    dist.barrier()
    out["status"] = ctx.status()
    return out


def main(out_dir):
    import kvmem_b200 as K
    from kvmem_b200.shard import LseGatherSelector, ShardCompute, ShardedSelector, ShardGeometry, page_ranges
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
        ids2, n2 = LseGatherSelector(ShardCompute(ctx)).select(desc, q, kc, geo, keep=[0, P - 1], budget=10)
        torch.cuda.synchronize()
        res = {"ids": [ids[l, : int(n[l])].tolist() for l in range(L)], "status": ctx.status(),
               "ids_lse": [ids2[l, : int(n2[l])].tolist() for l in range(L)]}
        if rank == 0:
            k_full = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
            full = K.RecallContext.make_kcache(k_full, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=P * B)
            _, mass = ctx.score_pages(desc, q, full, want_rows=False)
            rid, rn = ctx.select_topk(mass.view(L, P), [0, P - 1], 10)
            res["unsharded"] = [rid[l, : int(rn[l])].tolist() for l in range(L)]
        res["recall"] = sharded_recall_check(K, ctx, kb, qb, rank, world, local, dev, L, Hq, Hkv, D, B, P, T)
        res["recall_lse"] = sharded_recall_check(K, ctx, kb, qb, rank, world, local, dev, L, Hq, Hkv, D, B, P, T,
                                                 lse_gather=True)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
