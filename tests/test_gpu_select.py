"""GPU parity: kvm_select_topk against pick_scored_blocks (oracle and golden vectors).

Integer result: the selected page sets must be identical (bit-exact), ties
included, since the oracle ranks the same f32 scores.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")


def gpu_pick(ctx, scores_rows, keep, budget, signed=False):
    s = torch.tensor(np.asarray(scores_rows, np.float32), device="cuda")
    ids, n = ctx.select_topk(s, keep, budget, signed=signed)
    torch.cuda.synchronize()
    st = ctx.status()
    ids, n = ids.cpu().numpy(), n.cpu().numpy()
    return st, [ids[i, : n[i]].tolist() for i in range(len(n))]


@pytest.mark.parametrize("pages,budget,nrows", [(256, 18, 32), (512, 34, 64), (4096, 130, 8), (40000, 1000, 2),
                                                (7, 3, 5), (100, 200, 3), (1, 1, 1)])
def test_random_rows_match_oracle(ctx, pages, budget, nrows):
    rng = np.random.default_rng(pages + budget)
    scores = rng.random((nrows, pages)).astype(np.float32)
    scores[::2] = np.round(scores[::2] * 8) / 8  # many exact ties in every other row
    if nrows > 1:
        scores[1, :] = 0.25  # a row of equal scores: highest ids win
    keep = [0, pages - 1] if pages > 1 else [0]
    keep = keep[: min(len(keep), budget)]
    st, got = gpu_pick(ctx, scores, keep, budget)
    assert st == 0
    for r in range(nrows):
        rc, exp = O.pick_scored(pages, list(range(pages)), scores[r].astype(np.float64), keep, budget)
        assert rc == 0
        assert got[r] == exp.tolist(), f"row {r}"


def test_golden_picks(ctx):
    import kvmem_b200 as K
    golden = json.load(open(GOLDEN))
    for c in golden["pick"]:
        n = c["n"]
        if c["rc"] == 0:
            st, got = gpu_pick(ctx, [c["scores"]], c["mandatory"], c["budget"], c["signed"])
            assert st == 0 and got[0] == c["ids"]
        elif c["rc"] == 1:  # invalid candidate score: reported through the device status
            st, got = gpu_pick(ctx, [c["scores"]], c["mandatory"], c["budget"], c["signed"])
            assert st == K._abi.ERR_NONFINITE and got[0] == []
        else:  # mandatory pages exceed the budget: rejected before any launch
            with pytest.raises(K.KvmError) as e:
                gpu_pick(ctx, [c["scores"]], c["mandatory"], c["budget"], c["signed"])
            assert e.value.code == K._abi.ERR_BUDGET_EXCEEDED


def test_nonfinite_and_bad_keep(ctx):
    import kvmem_b200 as K
    s = np.ones((2, 16), np.float32)
    s[1, 3] = np.nan
    st, got = gpu_pick(ctx, s, [0], 4)
    assert st == K._abi.ERR_NONFINITE and got[0] == [0, 13, 14, 15] and got[1] == []
    assert ctx.status() == 0  # status was cleared by the read
    with pytest.raises(K.KvmError) as e:
        gpu_pick(ctx, s[:1], [16], 4)
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT


def test_pick_scored_blocks_mirror(ctx):
    import kvmem_b200 as K
    scores = torch.tensor([-.8, -.2, -.5], device="cuda")
    assert K.pick_scored_blocks(ctx, scores, [], 2, signed_scores=True) == [1, 2]
    with pytest.raises(ValueError):
        K.pick_scored_blocks(ctx, scores, [], 2)
    with pytest.raises(RuntimeError):
        K.pick_scored_blocks(ctx, torch.ones(5, device="cuda"), [0, 1, 2], 2)
