"""CPU tests: the oracle against the reference's own known answers and golden vectors.

The known answers restate kvmem/tests/graph_recall_test.cpp:22-106,242-253.
The golden vectors (tests/golden/reference_cases.json) were produced by the
reference's CPU code compiled from its sources (tests/golden/make_golden.py).
"""
import base64
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import util as U

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


def means_from_sums(sums, counts):
    inv = (np.float32(1.0) / np.asarray(counts, np.float32)).astype(np.float32)
    return (sums * inv[None, :, None]).astype(np.float32)


# ---------------------------------------------------------------- known answers

def test_frames_known_answers():
    f = O.query_score_frame(12, 4, 2, 0, 0, [2])
    assert f["score_mask"].tolist() == [1, 1, 1] and f["transport_mask"].tolist() == [1, 1, 0]
    s = O.query_score_frame(11, 4, 4, 1, 1, [0, 2])
    assert s["score_mask"].tolist() == [1, 1, 1] and s["transport_mask"].tolist() == [0, 0, 0]
    assert s["counts"][-1] == 3
    c = O.query_score_frame(12, 4, 2, 1, 1, [0, 2])
    assert c["score_mask"].tolist() == [0, 1, 0]


def test_page_softmax_known_answer():
    # graph_recall_test.cpp:32-56: keys {8,0},{0,4},{40,0} summed over 4 tokens.
    frame = O.query_score_frame(12, 4, 2, 0, 0, [2])
    means = means_from_sums(np.array([[[8, 0], [0, 4], [40, 0]]], np.float32), [4, 4, 4])
    q = np.array([[[2, 0], [0, 2]]], np.float32)  # one layer, two rows, one head
    res = O.meank_scores(means, q, [2], heads=1, kv_heads=1, dim=2, score_mask=frame["score_mask"])
    logits = [[4 / math.sqrt(2), 0, 20 / math.sqrt(2)], [0, 2 / math.sqrt(2), 0]]
    exp = [0.0, 0.0, 0.0]
    for line in logits:
        den = sum(math.exp(v) for v in line)
        for i in range(3):
            exp[i] += math.exp(line[i]) / den
    np.testing.assert_allclose(res, exp, atol=1e-12)
    assert abs(res.sum() - 2) < 1e-12
    assert res[1] > res[0]
    sm = frame["score_mask"].copy()
    sm[2] = 0
    wrong = O.meank_scores(means, q, [2], heads=1, kv_heads=1, dim=2, score_mask=sm)
    assert wrong[0] > wrong[1]
    empty = O.meank_scores(means, q, [2], heads=1, kv_heads=1, dim=2, score_mask=[0, 0, 0])
    assert empty.sum() == 0


def test_recall_fp16_known_answers():
    assert O.recall_fp16(1.00048828125) == 1.0
    assert O.recall_fp16(1.00146484375) == 1.001953125
    assert O.recall_fp16(2.0 ** -24) == 2.0 ** -24
    assert O.recall_fp16(2.0 ** -25) == 0.0
    with pytest.raises(ValueError):
        O.recall_fp16(65536.0)


def test_gqa_and_large_domain():
    # graph_recall_test.cpp:63-84
    means = np.array([[[1.0], [-1.0]], [[1.0], [-1.0]]], np.float32)
    frame = O.query_score_frame(2, 1, 1, 0, 0)
    q = np.array([[[1, -1]], [[2, -2]]], np.float32)
    res = O.meank_scores(means, q, [1, 1], heads=2, kv_heads=1, dim=1, score_mask=frame["score_mask"])
    np.testing.assert_allclose(res, [0.5, 0.5], atol=1e-12)
    for n in (8192, 8193, 32768, 32769):
        f = O.query_score_frame(n, 1, 1, 0, 0)
        s = O.meank_scores(np.ones((1, n, 1), np.float32), np.ones((1, 1, 1), np.float32), [1], heads=1,
                           kv_heads=1, dim=1, score_mask=f["score_mask"])
        assert abs(s[0] - 1 / n) < 1e-12 and abs(s[-1] - 1 / n) < 1e-12
        assert abs(s.sum() - 1) < 2e-12


def test_max_aggregation_and_signed_picker():
    # graph_recall_test.cpp:85-105
    means = np.array([[[1, 0], [0, 1], [-1, -1]]], np.float32)
    q = np.array([[[2, 0, 0, 2], [2, 0, 0, 2]]], np.float32)
    frame = O.query_score_frame(3, 1, 2, 0, 0)
    a, b, c = math.exp(math.sqrt(2)), 1.0, math.exp(-math.sqrt(2))
    mx, neg = a / (a + b + c), c / (a + b + c)
    mass = 2 * mx + neg
    s = O.meank_scores(means, q, [2], heads=2, kv_heads=1, dim=2, score_mask=frame["score_mask"], aggregation=1)
    np.testing.assert_allclose(s, [2 * mx / mass, 2 * mx / mass, 2 * neg / mass], atol=1e-12)
    rc, ids = O.pick_scored(3, [0, 1, 2], [-.8, -.2, -.5], [], 2, signed=True)
    assert rc == 0 and ids.tolist() == [1, 2]
    rc, _ = O.pick_scored(3, [0, 1, 2], [-.8, -.2, -.5], [], 2)
    assert rc == O.ERR_INVALID


def test_fixed_picker_media_rejects():
    # graph_recall_test.cpp:250-252
    rc, _ = O.pick_scored(6, [0, 3, 4, 5], [0, 1, 9, 8], [0, 3], 4, block_tokens=4, ranges=[(4, 9), (9, 13)])
    assert rc == O.ERR_RUNTIME


# ---------------------------------------------------------------- golden vectors

def test_golden_frames(golden):
    for c in golden["frames"]:
        f = O.query_score_frame(*c["args"], c["fixed"])
        assert f["score_mask"].tolist() == c["score_mask"]
        assert f["transport_mask"].tolist() == c["transport_mask"]
        assert f["counts"].tolist() == c["counts"]


def test_golden_recall_fp16(golden):
    for v, expected in golden["recall_fp16"]:
        value = float(v)
        if expected is None:
            with pytest.raises(ValueError):
                O.recall_fp16(value)
        else:
            assert O.recall_fp16(value) == expected, v


def test_golden_page_softmax(golden):
    for c in golden["page_softmax"]:
        L, P, R, D, Hq, Hkv = c["L"], c["P"], c["R"], c["D"], c["Hq"], c["Hkv"]
        sums = np.frombuffer(base64.b64decode(c["sums_f32_b64"]), np.float32).reshape(L, P, Hkv * D)
        q = np.frombuffer(base64.b64decode(c["q_f32_b64"]), np.float32).reshape(L, R, Hq * D)
        accepted = (P - 1) * c["block"] + c["counts"][-1]
        frame = O.query_score_frame(accepted, c["block"], c["budget"], c["sink"], c["recent"], c["fixed"])
        means = means_from_sums(sums, c["counts"])
        for agg, key in ((0, "expected_mean"), (1, "expected_max")):
            got = O.meank_scores(means, q, c["layer_rows"], heads=Hq, kv_heads=Hkv, dim=D,
                                 score_mask=frame["score_mask"], aggregation=agg)
            np.testing.assert_allclose(got, c[key], rtol=1e-12, atol=1e-15)


def test_golden_pick(golden):
    for c in golden["pick"]:
        rc, ids = O.pick_scored(c["n"], list(range(c["n"])), c["scores"], c["mandatory"], c["budget"],
                                signed=c["signed"])
        assert rc == c["rc"]
        if rc == 0:
            assert ids.tolist() == c["ids"]
    for c in golden["media_pick"]:
        rc, ids = O.pick_scored(6, c["cand"], c["scores"], c["mandatory"], c["budget"], block_tokens=4,
                                ranges=[(4, 9), (9, 13)])
        assert rc == c["rc"]
        if rc == 0:
            assert ids.tolist() == c["ids"]


def test_golden_residency(golden):
    for c in golden["residency"]:
        rc, d = O.plan_residency(c["resident"], c["selected"], c["force"])
        assert rc == c["rc"]
        if rc == 0:
            assert d["evict"].tolist() == c["evict"]
            assert d["retain"].tolist() == c["retain"]
            assert d["restore"].tolist() == c["restore"]


# ---------------------------------------------------------------- live reference (when built here)

@pytest.mark.skipif(O.ref() is None, reason="reference library not built (needs the reference sources)")
def test_live_reference_random_picks():
    rng = np.random.default_rng(3)
    for i in range(200):
        n = int(rng.integers(1, 600))
        scores = rng.random(n).astype(np.float32).astype(np.float64)
        if i % 2:
            scores = np.round(scores * 3) / 3
        budget = int(rng.integers(1, n + 2))
        mand = sorted(set(int(x) for x in rng.integers(0, n, int(rng.integers(0, 3)))))
        a = O.pick_scored(n, list(range(n)), scores, mand, budget)
        b = O.pick_scored(n, list(range(n)), scores, mand, budget, use_ref=True)
        assert a[0] == b[0]
        if a[0] == 0:
            assert a[1].tolist() == b[1].tolist()


# ---------------------------------------------------------------- per-token page mass oracle

def dense_page_mass(qv, kv, tokens, page, scale, softcap=0.0, bias=None):
    """Independent numpy restatement for one (layer, row): qv [Hq, D] f64, kv [T, Hkv, D] f64."""
    Hq, Hkv = qv.shape[0], kv.shape[1]
    G = Hq // Hkv
    pages = -(-tokens // page)
    out = np.zeros(pages)
    for h in range(Hq):
        lg = kv[:tokens, h // G, :] @ qv[h] * scale
        if softcap > 0:
            lg = softcap * np.tanh(lg / softcap)
        if bias is not None:
            lg = lg + bias[:tokens]
        p = np.exp(lg - lg.max())
        p /= p.sum()
        np.add.at(out, np.arange(tokens) // page, p / Hq)
    return out


@pytest.mark.parametrize("ktype", [U.F32, U.F16, U.BF16])
def test_page_mass_float_types_against_numpy(ktype):
    rng = np.random.default_rng(ktype)
    L, R, Hq, Hkv, D, T, page = 2, 2, 4, 2, 32, 50, 8
    kb = U.make_k(rng, ktype, L, 56, Hkv, D)
    qb = U.make_q(rng, U.F32, L, R, Hq, D)
    m = O.page_mass(qb, U.F32, kb, ktype, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                    page_tokens=page, scale=0.3, softcap=2.0 if ktype == U.F16 else 0.0)
    qv = qb.view(np.float32).reshape(L, R, Hq, D).astype(np.float64)
    if ktype == U.F32:
        kv = kb.view(np.float32)
    elif ktype == U.F16:
        kv = kb.view(np.float16).astype(np.float32)
    else:
        kv = (kb.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    kv = kv.reshape(L, 56, Hkv, D).astype(np.float64)
    for l in range(L):
        for r in range(R):
            exp = dense_page_mass(qv[l, r], kv[l], T, page, 0.3, 2.0 if ktype == U.F16 else 0.0)
            np.testing.assert_allclose(m[l, 0, r], exp, rtol=1e-12, atol=1e-15)
            assert abs(m[l, 0, r].sum() - 1) < 1e-12


def decode_blocks(raw, ktype, D):
    """Independent numpy decode of GGUF q8_0 / q4_0 / q5_0 rows."""
    nb = D // 32
    bb = U.BLOCK_BYTES[ktype]
    blk = raw.reshape(-1, nb, bb)
    d = blk[:, :, 0:2].copy().view(np.float16).astype(np.float64)[..., 0]
    if ktype == U.Q8_0:
        codes = blk[:, :, 2:].view(np.int8).astype(np.float64)
    elif ktype == U.Q4_0:
        qs = blk[:, :, 2:18]
        codes = np.concatenate([qs & 15, qs >> 4], axis=2).astype(np.float64) - 8
    else:
        qh = blk[:, :, 2:6].copy().view(np.uint32)[..., 0]
        qs = blk[:, :, 6:22]
        low = np.concatenate([qs & 15, qs >> 4], axis=2).astype(np.int64)
        high = (qh[..., None] >> np.arange(32)) & 1
        codes = (low | (high << 4)).astype(np.float64) - 16
    return (codes * d[..., None]).reshape(-1, D)


@pytest.mark.parametrize("ktype", [U.Q8_0, U.Q4_0, U.Q5_0])
def test_quant_decode_against_numpy(ktype):
    rng = np.random.default_rng(ktype + 10)
    D = 64
    raw = U.make_quant_rows(rng, ktype, 5, D)
    lib = O.lib()
    got = np.array([[lib.kvo_decode(ktype, raw[i].ctypes.data, d) for d in range(D)] for i in range(5)])
    np.testing.assert_array_equal(got, decode_blocks(raw, ktype, D))


def test_page_mass_groups_mask_and_empty_rows():
    rng = np.random.default_rng(2)
    L, R, Hq, Hkv, D, T, page = 1, 2, 4, 2, 32, 24, 8
    kb = U.make_k(rng, U.F16, L, T, Hkv, D)
    qb = U.make_q(rng, U.F16, L, R, Hq, D)
    mask = np.zeros((R, T), np.float32)
    mask[0, 5:9] = -np.inf
    mask[1, :] = -np.inf  # row 1 sees nothing -> NaN, as the reference's normaliser
    m = O.page_mass(qb, U.F16, kb, U.F16, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                    page_tokens=page, scale=0.2, groups=Hkv, mask=mask)
    assert m.shape == (1, 2, 2, 3)
    np.testing.assert_allclose(m[0, :, 0].sum(axis=1), [1, 1], atol=1e-12)
    assert np.isnan(m[0, :, 1]).all()


def test_meank_add_oracle_matches_numpy_sequential_sums():
    """The Mean-K producer restatement: per-page f32 sums of the decoded key
    elements added in token order, counts per page; checked against an
    independent numpy accumulation (f32 adds, f32 code*scale products)."""
    rng = np.random.default_rng(21)
    L, T, Hkv, D, B = 2, 150, 3, 64, 32
    P = -(-T // B)
    for kt in (U.F32, U.F16, U.BF16, U.Q8_0, U.Q4_0, U.Q5_0):
        kb = U.make_k(rng, kt, L, T, Hkv, D)
        sums = np.zeros((L, P, Hkv * D), np.float32)
        counts = np.zeros(P, np.uint32)
        for tok0, n in ((0, 40), (40, 1), (41, 1), (42, 108)):
            assert O.meank_add(sums, counts, kb, kt, layers=L, kv_heads=Hkv, dim=D, tok0=tok0, n=n,
                               page_tokens=B) == 0
        vals = U.decode_rows_f32(kb, kt, D)  # [L][T][Hkv][D] float32, code*scale rounded in f32
        ref = np.zeros_like(sums)
        for t in range(T):
            ref[:, t // B] = ref[:, t // B] + vals[:, t].reshape(L, Hkv * D)
        assert np.array_equal(sums, ref), kt
        assert counts.tolist() == [min(B, T - p * B) for p in range(P)]
    # a range past the table is refused
    assert O.meank_add(np.zeros((1, 2, 64), np.float32), np.zeros(2, np.uint32), U.make_k(rng, U.F16, 1, 100, 1, 64),
                       U.F16, layers=1, kv_heads=1, dim=64, tok0=60, n=10, page_tokens=32) == 1


def _random_graph(rng, n, block, accepted):
    starts = np.arange(n, dtype=np.uint64) * block
    rows = []
    for src in rng.choice(n + 3, size=rng.integers(0, n + 2), replace=False):
        edges = [(int(rng.integers(0, n + 2)) * block, float(rng.choice([0.0, rng.random()])))
                 for _ in range(rng.integers(0, 5))]
        rows.append((int(src) * block, int(rng.integers(0, 3)), edges))
    spans = None
    if rng.random() < 0.6:
        spans = []
        for _ in range(rng.integers(1, 4)):
            b = int(rng.integers(0, n * block))
            spans.append((b, b + int(rng.integers(1, 3 * block + 2)), bool(rng.random() < 0.7)))
    completed = int(rng.integers(0, n + 1)) * block
    return starts, dict(block=block, accepted=accepted, completed=completed, rows=rows, spans=spans)


def test_propagation_restatement_matches_reference():
    """propagate_query_scores (graph_recall.cpp:494-551): the C restatement
    against the compiled reference on random graphs, frames and scores."""
    if O.ref() is None:
        pytest.skip("reference library not built")
    rng = np.random.default_rng(5)
    for case in range(400):
        n = int(rng.integers(1, 30))
        block = int(rng.choice([1, 4, 64]))
        accepted = n * block
        starts, graph = _random_graph(rng, n, block, accepted)
        mask = (rng.random(n) < 0.85).astype(np.uint8)
        raw = rng.standard_normal(n) * rng.choice([0.01, 1.0, 30.0])
        raw[rng.random(n) < 0.2] = 0.0
        alpha = float(rng.choice([0.0, 0.2, 0.4, 1.0]))
        cross = float(rng.choice([0.25, 1.0, 0.0]))
        rc_o, out_o = O.propagate_scores(raw, starts, mask, accepted, graph, alpha, cross)
        rc_r, out_r = O.propagate_scores(raw, starts, mask, accepted, graph, alpha, cross, use_ref=True)
        assert rc_o == rc_r, (case, rc_o, rc_r)
        if rc_o == 0:
            np.testing.assert_allclose(out_o, out_r, rtol=1e-12, atol=1e-12 * max(1.0, np.abs(raw).sum()))


def test_propagation_known_answers_and_rejections():
    """Restated from the reference's graph_recall_test.cpp:160-187: three adjacent
    one-token pages, page 2 attends to page 0; explicit transport matrix."""
    starts = np.arange(3, dtype=np.uint64)
    graph = dict(block=1, accepted=3, completed=3, rows=[(2, 1, [(0, 1.0)])], spans=None)
    raw = np.array([0.8, -0.2, 0.4])
    rc, out = O.propagate_scores(raw, starts, np.ones(3, np.uint8), 3, graph, 0.4)
    assert rc == 0
    np.testing.assert_allclose(out, [0.8, -0.08, 0.28], atol=1e-12)
    assert abs(out.sum() - 1.0) < 1e-12
    rc, out = O.propagate_scores(raw, starts, np.ones(3, np.uint8), 3, graph, 0.0)
    assert rc == 0 and np.array_equal(out, raw)
    neg = np.array([-0.8, -0.2, -0.4])
    rc, out = O.propagate_scores(neg, starts, np.ones(3, np.uint8), 3, graph, 1.0)
    assert rc == 0 and np.array_equal(out, neg)
    rc, out = O.propagate_scores(raw, starts, np.array([1, 1, 0], np.uint8), 3, graph, 0.4)
    np.testing.assert_allclose(out, [0.72, -0.12, 0.4], atol=1e-12)
    assert O.propagate_scores([0, np.nan, 0], starts, np.ones(3, np.uint8), 3, graph, 0.0)[0] == 1
    assert O.propagate_scores([0, np.inf, 0], starts, np.ones(3, np.uint8), 3, graph, 0.4)[0] == 1
    assert O.propagate_scores(raw, starts, np.ones(3, np.uint8), 4, graph, 0.4)[0] == 1  # prefix mismatch


def test_lrfu_restatement_matches_reference():
    """LrfuHistory::preview (lrfu.hpp:57-79): bit-identical to the reference."""
    if O.ref() is None:
        pytest.skip("reference library not built")
    rng = np.random.default_rng(8)
    for case in range(300):
        n = int(rng.integers(1, 50))
        scores = rng.standard_normal(n) * rng.choice([0.001, 1.0, 100.0])
        scores[rng.random(n) < 0.1] = 0.0
        prev = rng.standard_normal(int(rng.integers(0, n + 5)))
        lam = float(rng.choice([0.0, 0.5, 1.0, 0.3]))
        frac = float(rng.choice([1.0, 0.9, 0.5, 0.01]))
        rc_o, a = O.lrfu_preview(scores, prev, lam, frac)
        rc_r, b = O.lrfu_preview(scores, prev, lam, frac, use_ref=True)
        assert rc_o == rc_r == 0
        assert np.array_equal(a, b), case
    assert O.lrfu_preview([1.0, np.nan], [], 0.5, 0.9)[0] == 1


@pytest.mark.parametrize("kt", [U.Q8_0, U.Q4_0])
def test_restore_k_oracle_matches_numpy(kt):
    """Raw-K restore transform (stagein.cu:104-234): dequant -> NeoX RoPE -> FWHT ->
    requant. Bit-exact against the numpy restatement without RoPE; with RoPE the
    sin / cos of the two libraries may differ in the last bits, so requantised
    values stay within one quantisation step and nearly all codes agree."""
    rng = np.random.default_rng(12 + kt)
    tokens, n_head, dim = 9, 4, 128
    theta = (10000.0 ** (-np.arange(0, dim, 2) / dim)).astype(np.float32)
    kb = U.make_k(rng, kt, 1, tokens, n_head, dim).reshape(-1)
    for n_rot, nrot in ((0, 0), (0, 64), (0, 128), (0, 512), (dim, 256), (64, 128), (dim, 0)):
        rc, got = O.restore_k(kt, kb, tokens=tokens, n_head=n_head, dim=dim, n_rot=n_rot, pos0=1000, theta=theta,
                              nrot=nrot)
        assert rc == 0
        exp = U.restore_k_numpy(kt, kb, tokens, n_head, dim, n_rot, 1000, theta, nrot)
        if n_rot == 0:
            assert np.array_equal(got, exp), (n_rot, nrot)
        else:
            a = U.decode_rows_f32(got.reshape(tokens * n_head, -1), kt, dim)
            b = U.decode_rows_f32(exp.reshape(tokens * n_head, -1), kt, dim)
            step = np.abs(U.decode_rows_f32(exp.reshape(tokens * n_head, -1), kt, dim)).max() / (7 if kt == U.Q4_0 else 100)
            assert np.abs(a - b).max() <= step
            assert np.mean(got == exp) > 0.97
    assert O.restore_k(kt, kb, tokens=tokens, n_head=n_head, dim=dim, nrot=96)[0] == 1
