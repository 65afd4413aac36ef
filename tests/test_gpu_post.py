"""GPU parity: post-scoring fusion on the device (propagation over the
attention-feedback graph, LRFU preview) and the whole Query chain
Mean-K scores -> propagation -> LRFU -> signed top-k, against the oracle
(C restatements pinned to the compiled reference in tests/test_oracle.py).
Scores are f32 on the device, double in the oracle: |gpu - oracle| <=
1e-6 * |oracle| + 1e-6 * sum|raw|; selections equal wherever the gap at the
budget boundary exceeds 1e-3 relative (the north-star rule)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_oracle import _random_graph

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.device("cuda", 0))


def test_propagation_random_graphs(ctx):
    import kvmem_b200 as K
    rng = np.random.default_rng(31)
    checked = 0
    for case in range(150):
        n = int(rng.integers(1, 60))
        block = int(rng.choice([1, 16, 64]))
        starts, graph = _random_graph(rng, n, block, n * block)
        mask = (rng.random(n) < 0.85).astype(np.uint8)
        raw = (rng.standard_normal(n) * rng.choice([0.01, 1.0, 30.0])).astype(np.float32)
        raw[rng.random(n) < 0.2] = 0.0
        alpha = float(rng.choice([0.0, 0.2, 0.4, 1.0]))
        cross = float(rng.choice([0.25, 1.0, 0.0]))
        rc, exp = O.propagate_scores(raw.astype(np.float64), starts, mask, n * block, graph, alpha, cross)
        if rc != 0:
            with pytest.raises(K.KvmError):
                ctx.propagate_scores(_dev(raw), starts, mask, n * block, graph, alpha=alpha, cross=cross)
            continue
        got = ctx.propagate_scores(_dev(raw), starts, mask, n * block, graph, alpha=alpha, cross=cross)
        torch.cuda.synchronize()
        ctx.check_status("propagate")
        tol = 1e-6 * np.abs(exp) + 1e-6 * max(1.0, float(np.abs(raw).sum()))
        assert np.all(np.abs(got.cpu().numpy() - exp) <= tol), case
        checked += 1
    assert checked > 100


def test_propagation_known_answers(ctx):
    """graph_recall_test.cpp:160-185 restated, on the device."""
    starts = [0, 1, 2]
    graph = dict(block=1, accepted=3, completed=3, rows=[(2, 1, [(0, 1.0)])], spans=None)
    got = ctx.propagate_scores(_dev([0.8, -0.2, 0.4]), starts, [1, 1, 1], 3, graph, alpha=0.4).cpu().numpy()
    np.testing.assert_allclose(got, [0.8, -0.08, 0.28], atol=1e-7)
    got = ctx.propagate_scores(_dev([0.8, -0.2, 0.4]), starts, [1, 1, 0], 3, graph, alpha=0.4).cpu().numpy()
    np.testing.assert_allclose(got, [0.72, -0.12, 0.4], atol=1e-7)
    neg = np.array([-0.8, -0.2, -0.4], np.float32)
    assert np.array_equal(ctx.propagate_scores(_dev(neg), starts, [1, 1, 1], 3, graph, alpha=1.0).cpu().numpy(), neg)


def test_propagation_rejections(ctx):
    import kvmem_b200 as K
    graph = dict(block=4, accepted=12, completed=12, rows=[], spans=None)
    with pytest.raises(K.KvmError) as e:  # the graph belongs to another accepted prefix
        ctx.propagate_scores(_dev([1, 0, 1]), [0, 4, 8], [1, 1, 1], 16, graph)
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
    with pytest.raises(K.KvmError) as e:  # duplicate start
        ctx.propagate_scores(_dev([1, 0, 1]), [0, 4, 4], [1, 1, 1], 12, graph)
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
    with pytest.raises(K.KvmError) as e:  # alpha outside [0, 1]
        ctx.propagate_scores(_dev([1, 0, 1]), [0, 4, 8], [1, 1, 1], 12, graph, alpha=1.5)
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
    ctx.propagate_scores(_dev([1, np.nan, 1]), [0, 4, 8], [1, 1, 1], 12, graph)
    torch.cuda.synchronize()
    with pytest.raises(K.KvmError) as e:
        ctx.check_status("propagate")
    assert e.value.code == K._abi.ERR_NONFINITE


@pytest.mark.parametrize("fraction", [1.0, 0.9, 0.5, 0.01])
def test_lrfu_preview_matches_oracle(ctx, fraction):
    rng = np.random.default_rng(int(fraction * 100))
    for case in range(40):
        n = int(rng.integers(1, 3000))
        s = (rng.standard_normal(n) * rng.choice([0.001, 1.0, 100.0])).astype(np.float32)
        s[rng.random(n) < 0.1] = 0.0
        s[rng.random(n) < 0.05] = s[0]  # ties
        prev = rng.standard_normal(int(rng.integers(0, n + 10))).astype(np.float32)
        lam = float(rng.choice([0.0, 0.5, 1.0]))
        rc, exp = O.lrfu_preview(s.astype(np.float64), prev.astype(np.float64), lam, fraction)
        assert rc == 0
        got = ctx.lrfu_preview(_dev(s), _dev(prev) if len(prev) else None, lam=lam, fraction=fraction)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), exp.astype(np.float32), rtol=2e-7, atol=1e-30)


def test_query_chain_selects_like_the_oracle(ctx):
    """Mean-K page softmax -> propagation -> LRFU preview -> signed top-k, all on
    the device, against the same chain in the oracle."""
    import kvmem_b200 as K
    from tests.test_gpu_meank import means_from_sums
    rng = np.random.default_rng(77)
    L, P, Hkv, Hq, D, R, B = 2, 96, 2, 8, 64, 2, 64
    budget = 12
    for case in range(6):
        sums = (rng.standard_normal((L, P, Hkv * D)) * 4).astype(np.float32)
        counts = np.full(P, B, np.uint32)
        q = rng.standard_normal((L, R, Hq * D)).astype(np.float32)
        frame = O.query_score_frame(P * B, B, budget, 1, 1)
        mask = frame["score_mask"]
        raw_o = O.meank_scores(means_from_sums(sums, counts), q, np.full(L, R, np.uint32), heads=Hq, kv_heads=Hkv,
                               dim=D, score_mask=mask, aggregation=0, scale=1 / np.sqrt(D))
        starts, graph = _random_graph(rng, P, B, P * B)
        graph["completed"] = P * B
        tmask = frame["transport_mask"]
        rc, prop_o = O.propagate_scores(raw_o, starts, tmask, P * B, graph, 0.2, 0.25)
        assert rc == 0
        prev = (rng.random(P) * 0.02).astype(np.float32)
        rc, cand_o = O.lrfu_preview(prop_o, prev.astype(np.float64), 0.5, 0.9)
        assert rc == 0
        keep = [0, P - 1]  # the sink and recent pages
        rc, ids_o = O.pick_scored(P, list(range(P)), cand_o, keep, budget, signed=True)
        assert rc == 0
        out = ctx.meank_score(_dev(sums), torch.from_numpy(counts.view(np.int32)).cuda(), _dev(q), [R] * L, mask,
                              q_heads=Hq, kv_heads=Hkv, head_dim=D, aggregation=0, scale=float(1 / np.sqrt(D)))
        prop = ctx.propagate_scores(out, [int(x) for x in starts], tmask, P * B, graph, alpha=0.2, cross=0.25)
        cand = ctx.lrfu_preview(prop, _dev(prev), lam=0.5, fraction=0.9)
        ids, n = ctx.select_topk(cand.view(1, P), keep, budget, signed=True)
        torch.cuda.synchronize()
        ctx.check_status("query chain")
        got = sorted(ids[0, : int(n[0])].tolist())
        order = np.argsort(-cand_o, kind="stable")
        free = [p for p in order if p not in set(keep)]
        k = budget - len(set(keep))
        gap = abs(cand_o[free[k - 1]] - cand_o[free[k]]) / max(abs(cand_o[free[k - 1]]), 1e-30)
        if gap > 1e-3:
            assert got == sorted(ids_o), case
