"""GPU parity of page-range sharded selection (kvm_shard_*), ranks emulated on one GPU.

Both exchanges are covered: statistics + candidates (kvm_shard_score_partial ...
kvm_shard_merge) and the one-collective page-LSE gather (kvm_shard_page_lse +
kvm_page_mass_from_lse + kvm_select_topk), which must reproduce the unsharded
masses bit for bit.

Each emulated rank has its own context (its page LSE stays in its workspace
between the partial and finish passes); the all-gathers are torch.stack. The
sharded masses must equal the unsharded kvm_score_pages masses (fp32 rounding
only: 1e-5 relative) and the selection must equal the FP64 oracle's
pick_scored_blocks wherever the score gap at the k-th boundary exceeds 1e-3
relative (the north-star rule); fp16 histories carry needle pages so their
boundary gaps are wide, q8_0 rows are compared where the gap rule allows.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import util as U

pytestmark = pytest.mark.gpu


def boundary_gap(mass, keep, k):
    s = np.sort(np.delete(mass, keep))[::-1]
    return (s[k - 1] - s[k]) / max(s[k - 1], 1e-30) if len(s) > k else 1.0


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("ktype", [U.F16, U.Q8_0])
def test_emulated_ranks_match_unsharded_and_oracle(world, ktype):
    import kvmem_b200 as K
    from kvmem_b200.shard import ShardCompute, ShardGeometry, page_ranges
    rng = np.random.default_rng(world * 10 + ktype)
    L, Hq, Hkv, D, B, P = 2, 24, 4, 256, 64, 37
    T = P * B - 17
    qb = U.make_q(rng, U.F32, L, 1, Hq, D)
    qdir = qb.view(np.float32).reshape(L, 1, Hq, D)[:, 0].reshape(L, Hkv, Hq // Hkv, D).mean(axis=2)
    qdir /= np.sqrt((qdir ** 2).mean(axis=-1, keepdims=True))
    kb = U.make_k(rng, ktype, L, P * B, Hkv, D, needle_pages=(3, 11, 17, 20, 29, 33), page=B, q_dir=qdir / np.sqrt(D))
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, 1, Hq, D)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=B)
    q = K.RecallContext.make_query(q_d, 1)
    full = K.RecallContext.make_kcache(k_d, ktype, kv_heads=Hkv, head_dim=D, capacity_tokens=P * B)
    ctx0 = K.RecallContext(0)
    _, ref_mass = ctx0.score_pages(desc, q, full, want_rows=False)
    keep, budget = [0, P - 1], 8
    ref_ids, ref_n = ctx0.select_topk(ref_mass.view(L, P), keep, budget)

    page_bytes = B * Hkv * U.row_bytes(ktype, D)
    ranges = page_ranges(P, world)
    ctxs = [K.RecallContext(0) for _ in range(world)]
    comps = [ShardCompute(c) for c in ctxs]
    geos, kcs = [], []
    for r, (p0, p1) in enumerate(ranges):
        geos.append(ShardGeometry(layers=L, rows=1, q_heads=Hq, kv_heads=Hkv, groups=1, total_pages=P, page0=p0,
                                  local_pages=p1 - p0))
        kcs.append(K.RecallContext.make_kcache(k_d, ktype, kv_heads=Hkv, head_dim=D, capacity_tokens=(p1 - p0) * B,
                                               layer_stride=full.layer_stride,
                                               data_ptr=k_d.data_ptr() + p0 * page_bytes))
    stats = torch.stack([comps[r].partial(desc, q, kcs[r], geos[r]) for r in range(world)])
    gstats = comps[0].merge_stats(stats, world, geos[0])
    masses = [comps[r].finish(desc, geos[r], gstats) for r in range(world)]
    mass = torch.cat(masses, dim=1)
    torch.cuda.synchronize()
    np.testing.assert_allclose(mass.cpu().numpy(), ref_mass.view(L, P).cpu().numpy(), rtol=1e-5, atol=1e-9)
    kc = budget - len(keep)
    cands = [comps[r].candidates(masses[r], geos[r], keep, kc) for r in range(world)]
    gs = torch.stack([c[0] for c in cands])
    gi = torch.stack([c[1] for c in cands])
    ids, n = comps[0].merge(gs, gi, world, geos[0], keep, kc, budget)
    torch.cuda.synchronize()
    for c in ctxs + [ctx0]:
        assert c.status() == 0
    exp = O.page_mass(qb, U.F32, kb, ktype, layers=L, rows=1, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=B, scale=float(np.float32(1) / np.sqrt(np.float32(D))))[:, 0, 0]
    ids, n = ids.cpu().numpy(), n.cpu().numpy()
    ref_ids, ref_n = ref_ids.cpu().numpy(), ref_n.cpu().numpy()
    compared = 0
    for l in range(L):
        if boundary_gap(exp[l], keep, kc) <= 1e-3:
            continue
        compared += 1
        rc, want = O.pick_scored(P, list(range(P)), exp[l], keep, budget)
        assert ids[l, : n[l]].tolist() == want.tolist()
        assert ref_ids[l, : ref_n[l]].tolist() == want.tolist()
    if ktype == U.F16:
        assert compared == L

    # The one-collective exchange: each rank's page LSE (kvm_shard_page_lse), the ranges side
    # by side, whole-row masses (kvm_page_mass_from_lse): the same LSE values and the same
    # normaliser as the unsharded call, so the masses and the top-k are identical to it.
    lses = [comps[r].page_lse(desc, q, kcs[r], geos[r]) for r in range(world)]
    full_lse = torch.cat(lses, dim=-1)
    mass2 = comps[0].mass_from_lse(desc, geos[0], full_lse)
    ids2, n2 = comps[0].select_topk(mass2, keep, budget)
    torch.cuda.synchronize()
    assert ctxs[0].status() == 0
    np.testing.assert_array_equal(mass2.cpu().numpy(), ref_mass.view(L, P).cpu().numpy())
    ids2, n2 = ids2.cpu().numpy(), n2.cpu().numpy()
    for l in range(L):
        assert ids2[l, : n2[l]].tolist() == ref_ids[l, : ref_n[l]].tolist()
