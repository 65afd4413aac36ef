"""GPU parity: kvm_select_topk_media against the reference's own pick_scored_blocks.

The device picker with media groups is compared with KvMemStore::pick_scored_blocks
compiled from the reference's sources (oracle/_ref/libkvref.so) on random rows:
media ranges that chain, nest, touch without overlapping, start mid-page or run
past the history; tied scores; keep pages inside groups; budgets that force
groups to be skipped. Integer result: the page sets must be identical.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")


def ref_pick(n, scores, keep, budget, block, ranges, signed=False):
    if O.ref() is None:
        pytest.fail("oracle/_ref/libkvref.so is missing (make -C oracle ref)")
    return O.pick_scored(n, list(range(n)), np.asarray(scores, np.float64), keep, budget, signed=signed,
                         block_tokens=block, ranges=ranges, use_ref=True)


def gpu_pick(ctx, rows, keep, budget, block, ranges, signed=False):
    s = torch.tensor(np.asarray(rows, np.float32), device="cuda")
    ids, n = ctx.select_topk_media(s, keep, budget, block_tokens=block, media_ranges=ranges, signed=signed)
    torch.cuda.synchronize()
    st = ctx.status()
    ids, n = ids.cpu().numpy(), n.cpu().numpy()
    return st, [ids[i, : n[i]].tolist() for i in range(len(n))]


def random_ranges(rng, pages, block, count):
    out = []
    for _ in range(count):
        a = int(rng.integers(0, pages * block))
        ln = int(rng.integers(1, 6 * block))
        out.append((a, min(a + ln, pages * block + 3 * block)))
    return out


@pytest.mark.parametrize("pages,block,budget,nranges,nrows",
                         [(64, 16, 12, 6, 8), (512, 256, 34, 20, 16), (4096, 256, 130, 60, 4),
                          (300, 64, 40, 0, 4), (16384, 64, 200, 150, 2), (9, 4, 3, 4, 6)])
def test_random_rows_match_reference(ctx, pages, block, budget, nranges, nrows):
    rng = np.random.default_rng(pages + budget + nranges)
    ranges = random_ranges(rng, pages, block, nranges)
    if nranges:
        ranges.append((3 * block, 3 * block))  # empty range: no group
        ranges.append((5 * block + 1, 7 * block - 1))  # starts and ends mid-page
        ranges.append((7 * block, 9 * block))  # touches the previous span: a separate group
    scores = rng.random((nrows, pages)).astype(np.float32)
    scores[::2] = np.round(scores[::2] * 8) / 8  # many exact ties
    keep = [0, pages - 1]
    rc, _ = ref_pick(pages, scores[0], keep, budget, block, ranges)
    if rc != 0:  # the keep groups alone overflow this budget: keep page 0 only
        keep = [0]
    st, got = gpu_pick(ctx, scores, keep, budget, block, ranges)
    assert st == 0
    for r in range(nrows):
        rc, exp = ref_pick(pages, scores[r], keep, budget, block, ranges)
        assert rc == 0
        assert got[r] == exp.tolist(), f"row {r}"


def test_signed_scores_and_skipped_groups(ctx):
    """A large group ranked first that does not fit is skipped for good; smaller
    groups and single pages behind it still fill the budget."""
    pages, block = 40, 8
    ranges = [(0, 8 * 10), (8 * 20, 8 * 23), (8 * 30 + 4, 8 * 31 + 2)]  # pages 0-9, 20-22, 30
    rng = np.random.default_rng(3)
    rows = rng.standard_normal((4, pages)).astype(np.float32)
    rows[:, 5] = 50.0  # best page inside the 10-page group
    rows[:, 21] = 40.0  # second best inside the 3-page group
    for budget in (4, 9, 10, 13, 14, 40):
        st, got = gpu_pick(ctx, rows, [39], budget, block, ranges, signed=True)
        assert st == 0
        for r in range(len(rows)):
            rc, exp = ref_pick(pages, rows[r], [39], budget, block, ranges, signed=True)
            assert rc == 0 and got[r] == exp.tolist(), (budget, r)


def test_golden_media_picks(ctx):
    """The golden cases whose candidates are every page (graph_recall_test.cpp:242-253 shape)."""
    golden = json.load(open(GOLDEN))
    used = 0
    for c in golden["media_pick"]:
        if c["cand"] != list(range(len(c["scores"]))) or c["rc"] != 0:
            continue
        st, got = gpu_pick(ctx, [c["scores"]], c["mandatory"], c["budget"], 4, [(4, 9), (9, 13)])
        assert st == 0 and got[0] == c["ids"]
        used += 1
    assert used >= 1


def test_rejections(ctx):
    import kvmem_b200 as K
    s = torch.rand((2, 20), device="cuda")
    with pytest.raises(K.KvmError) as e:  # the keep page's group (pages 0-7) exceeds the budget
        ctx.select_topk_media(s, [2], 5, block_tokens=4, media_ranges=[(0, 32)])
    assert e.value.code == K._abi.ERR_BUDGET_EXCEEDED
    with pytest.raises(K.KvmError) as e:
        ctx.select_topk_media(s, [20], 5, block_tokens=4, media_ranges=[])
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
    with pytest.raises(K.KvmError) as e:
        ctx.select_topk_media(torch.rand((1, 16385), device="cuda"), [], 5, block_tokens=4, media_ranges=[])
    assert e.value.code == K._abi.ERR_LENGTH
    bad = torch.rand((1, 20), device="cuda")
    bad[0, 3] = -1.0
    ids, n = ctx.select_topk_media(bad, [], 5, block_tokens=4, media_ranges=[])
    torch.cuda.synchronize()
    assert ctx.status() == K._abi.ERR_NONFINITE and int(n[0]) == 0  # reading the status clears it


def test_calls_on_two_streams_keep_their_own_groups(ctx):
    """Back-to-back calls on two streams with different media ranges: the second call's
    group table must not overwrite the first's while the first kernel may still read it."""
    pages, block, budget = 4096, 64, 130
    rng = np.random.default_rng(17)
    rows = rng.random((8, pages)).astype(np.float32)
    ranges_a = random_ranges(rng, pages, block, 80)
    ranges_b = random_ranges(rng, pages, block, 80)
    s = torch.tensor(rows, device="cuda")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    outs = []
    for _ in range(3):
        with torch.cuda.stream(s1):  # outputs allocated and written on s1
            ia, na = ctx.select_topk_media(s, [0], budget, block_tokens=block, media_ranges=ranges_a, stream=s1)
        with torch.cuda.stream(s2):
            ib, nb = ctx.select_topk_media(s, [0], budget, block_tokens=block, media_ranges=ranges_b, stream=s2)
        outs.append((ia, na, ib, nb))
    torch.cuda.synchronize()
    assert ctx.status() == 0
    for ia, na, ib, nb in outs:
        ia, na, ib, nb = ia.cpu().numpy(), na.cpu().numpy(), ib.cpu().numpy(), nb.cpu().numpy()
        for r in range(len(rows)):
            rc, exp_a = ref_pick(pages, rows[r], [0], budget, block, ranges_a)
            rc2, exp_b = ref_pick(pages, rows[r], [0], budget, block, ranges_b)
            assert rc == 0 and rc2 == 0
            assert ia[r, : na[r]].tolist() == exp_a.tolist()
            assert ib[r, : nb[r]].tolist() == exp_b.tolist()
