"""GPU: layerwise tile accumulation (kvm_layerwise_accumulate / kvm_layerwise_finish).

The layerwise recall scores a prefill's query rows of one layer in tiles against one
frozen frame and sums the tiles' page masses (kvmem/src/host/layerwise_selection.cpp:
layerwise_tile_scores :32-75, LayerwiseQuerySelection::accumulate :283-296 and finish
:298-309). Tiles here are scored on the device with kvm_meank_score (whose weight over
one layer is 1 / query heads, summed over the rows, as PageSoftmaxCuda::score_current_layer)
over Mean-K records of half pages (two per transport page) and of whole pages, then:

* the device accumulation equals, bit for bit, the reference's own layerwise_tile_scores
  of each tile's masses summed in tile order, and with keep_halves its
  layerwise_max_page_scores (the compiled reference, oracle/_ref/libkvref.so);
* the tiles sum to the scores of all rows in one call (the reference's own check,
  kvmem/tests/layerwise_scoring_test.cpp:95-110), within the scorer's qualification
  bound 2e-6 + 3e-5 * expected;
* a tile that fails the reference's checks (a NaN, a negative half, mass on a page
  outside the score mask) sets the context status and adds nothing.
"""
import numpy as np
import pytest
import torch

import kvmem_b200 as K
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PAGE, HALF = 8, 4


def _setup(rng, pages, halves, layers=1, hq=8, hkv=2, dim=128, rows=96):
    kw = hkv * dim
    slots = pages * halves
    sums = (rng.standard_normal((layers, slots, kw)) * 3).astype(np.float32)
    counts = np.full(slots, PAGE // halves, np.uint32)
    q = rng.standard_normal((layers, rows, hq * dim)).astype(np.float32)
    return sums, counts, q


def _tile(ctx, sums_d, counts_d, q, first, n, mask_slots, hq, hkv, dim):
    dev = sums_d.device
    qt = torch.from_numpy(np.ascontiguousarray(q[:, first:first + n])).to(dev)
    return ctx.meank_score(sums_d, counts_d, qt, [n], mask_slots, q_heads=hq, kv_heads=hkv, head_dim=dim)


@pytest.mark.parametrize("halves,keep", [(2, True), (2, False), (1, False)], ids=["halves_max", "halves_sum", "pages"])
def test_tiles_match_reference_and_sum_to_the_whole(ctx, halves, keep):
    rng = np.random.default_rng(halves * 10 + keep)
    pages, hq, hkv, dim, rows = 200, 8, 2, 128, 96
    sums, counts, q = _setup(rng, pages, halves, hq=hq, hkv=hkv, dim=dim, rows=rows)
    frame = O.query_score_frame(pages * PAGE, PAGE, 16, 1, 1, [0, pages - 1], use_ref=True)
    assert len(frame["starts"]) == pages
    mask = np.asarray(frame["score_mask"], np.uint8)
    mask_slots = np.repeat(mask, halves)
    dev = torch.device("cuda", 0)
    sums_d = torch.from_numpy(sums).to(dev)
    counts_d = torch.from_numpy(counts.view(np.int32)).to(dev)
    mask_d = torch.from_numpy(mask).to(dev)
    accum = torch.zeros(pages * (2 if keep else 1), dtype=torch.float64, device=dev)
    want = np.zeros(pages * (2 if keep else 1), np.float64)
    for first, n in [(0, 40), (40, 17), (57, rows - 57)]:
        t = _tile(ctx, sums_d, counts_d, q, first, n, mask_slots, hq, hkv, dim)
        ctx.layerwise_accumulate(t, mask_d, accum, halves=halves, keep_halves=keep)
        want += O.ref_layerwise_tile_scores(frame, PAGE, PAGE // halves, keep, t.cpu().numpy().astype(np.float64))
    got = ctx.layerwise_finish(accum, pages, keep_halves=keep)
    torch.cuda.synchronize()
    ctx.check_status("layerwise")
    final = O.ref_layerwise_max_page_scores(want) if keep else want
    np.testing.assert_array_equal(accum.cpu().numpy(), want)
    np.testing.assert_array_equal(got.cpu().numpy(), final.astype(np.float32))
    # the tiles sum to all rows scored at once
    whole = _tile(ctx, sums_d, counts_d, q, 0, rows, mask_slots, hq, hkv, dim).cpu().numpy().astype(np.float64)
    whole = whole.reshape(pages, halves)
    acc = accum.cpu().numpy().reshape(pages, -1)
    whole_slots = whole if keep else whole.sum(axis=1, keepdims=True)
    bad = np.abs(acc - whole_slots) > 2e-6 + 3e-5 * np.abs(whole_slots)
    assert not bad.any(), f"{int(bad.sum())} slots: tiles do not sum to the whole"
    assert abs(acc.sum() - rows) < rows * 2e-5  # every row's probability mass is 1


def test_invalid_tiles_add_nothing(ctx):
    pages = 50
    frame = O.query_score_frame(pages * PAGE, PAGE, 16, 1, 1, [0, pages - 1], use_ref=True)
    mask = np.asarray(frame["score_mask"], np.uint8)
    dev = torch.device("cuda", 0)
    mask_d = torch.from_numpy(mask).to(dev)
    good = np.where(np.repeat(mask, 2) > 0, 0.01, 0.0).astype(np.float32)
    accum = torch.zeros(pages * 2, dtype=torch.float64, device=dev)
    ctx.layerwise_accumulate(torch.from_numpy(good).to(dev), mask_d, accum, halves=2, keep_halves=True)
    torch.cuda.synchronize()
    assert ctx.status() == 0
    before = accum.cpu().numpy().copy()
    cases = []
    nan = good.copy()
    nan[7] = np.nan
    cases.append((nan, K._abi.ERR_INVALID_ARGUMENT))  # the half sum is not finite
    neg = good.copy()
    neg[9] = -1e-3
    cases.append((neg, K._abi.ERR_INVALID_ARGUMENT))  # a negative half
    outside = good.copy()
    outside[0] = 0.5  # page 0 (sink) is outside the score mask
    assert mask[0] == 0
    cases.append((outside, K._abi.ERR_INVALID_ARGUMENT))
    for tile, code in cases:
        ctx.layerwise_accumulate(torch.from_numpy(tile).to(dev), mask_d, accum, halves=2, keep_halves=True)
        torch.cuda.synchronize()
        assert ctx.status() == code
        np.testing.assert_array_equal(accum.cpu().numpy(), before)
    # whole-page records: a NaN fails the accumulate checks (the reference's InvalidPlan)
    one = torch.zeros(pages, dtype=torch.float64, device=dev)
    t = np.where(mask > 0, 0.02, 0.0).astype(np.float32)
    t[3] = np.nan
    ctx.layerwise_accumulate(torch.from_numpy(t).to(dev), mask_d, one, halves=1)
    torch.cuda.synchronize()
    assert ctx.status() == K._abi.ERR_INVALID_PLAN
    assert float(one.abs().sum()) == 0.0
    with pytest.raises(K.KvmError):  # keeping halves needs two records per page
        ctx.layerwise_accumulate(torch.from_numpy(t).to(dev), mask_d, one, halves=1, keep_halves=True)
