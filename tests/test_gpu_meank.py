"""GPU parity: kvm_meank_score (Mean-K page softmax) against the FP64 oracle and
the reference's golden vectors.

Restates the reference's GPU qualification (kvmem/tests/graph_recall_cuda_test.cpp:16-59):
its shapes, its operand formulas, tolerance |d| <= 2e-6 + 3e-5 * expected per page,
the softmax mass equal to `rows` within rows * 2e-5, and the borrowed workspace.
"""
import base64
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")


def within(actual, expected):
    actual, expected = np.asarray(actual), np.asarray(expected)
    err = np.abs(actual - expected)
    return bool(np.all(np.isfinite(actual)) and np.all(err <= 2e-6 + expected * 3e-5)), float(err.max(initial=0))


def means_from_sums(sums, counts):
    inv = (np.float32(1.0) / np.asarray(counts, np.float32)).astype(np.float32)
    return (sums * inv[None, :, None]).astype(np.float32)


@pytest.mark.parametrize("agg", [0, 1])
@pytest.mark.parametrize("shape", [(7, 129, 256, 8, 2), (8192, 2, 64, 4, 1), (8193, 2, 64, 4, 1),
                                   (32769, 1, 64, 2, 1)])
def test_reference_qualification_shapes(shape, agg):
    import kvmem_b200 as K
    blocks, rows, dim, qheads, kvheads = shape
    layers = 2
    kw, qw = kvheads * dim, qheads * dim
    b = np.arange(blocks)[:, None]
    d = np.arange(kw)[None, :]
    sums = np.stack([((b * 13 + d * 7 + l * 11) % 101 - 50).astype(np.float32) / 16 for l in range(layers)])
    counts = np.full(blocks, 4, np.uint32)
    q = ((np.arange(layers * rows * qw) * 17) % 127 - 63).astype(np.float32).reshape(layers, rows, qw) / 32
    frame = O.query_score_frame(blocks * 4, 4, 3, 1, 1, [0, blocks - 1])
    expected = O.meank_scores(means_from_sums(sums, counts), q, [rows, rows], heads=qheads, kv_heads=kvheads,
                              dim=dim, score_mask=frame["score_mask"], aggregation=agg)
    dev = torch.device("cuda", 0)
    sums_d = torch.from_numpy(sums).to(dev)
    counts_d = torch.from_numpy(counts.view(np.int32)).to(dev)
    q_d = torch.from_numpy(q).to(dev)
    scorer = K.PageSoftmaxCuda(0)
    actual = scorer.score(sums_d, counts_d, q_d, [rows, rows], frame, agg, q_heads=qheads, kv_heads=kvheads,
                          head_dim=dim)
    ok, worst = within(actual, expected)
    assert ok, f"CUDA page softmax differs from represented-input FP64 oracle (worst {worst:.3g})"
    assert abs(sum(actual) - rows) <= rows * 2e-5, "CUDA softmax mass was lost"
    if blocks == 7:  # borrowed workspace
        ws = torch.empty(1 << 22, dtype=torch.uint8, device=dev)
        planned = K.PageSoftmaxCuda(0, workspace=ws).score(sums_d, counts_d, q_d, [rows, rows], frame, agg,
                                                            q_heads=qheads, kv_heads=kvheads, head_dim=dim)
        ok, worst = within(planned, expected)
        assert ok, "planned workspace differs from FP64 oracle"
        tiny = K.PageSoftmaxCuda(0, workspace=torch.empty(1024, dtype=torch.uint8, device=dev))
        with pytest.raises(OverflowError):
            tiny.score(sums_d, counts_d, q_d, [rows, rows], frame, agg, q_heads=qheads, kv_heads=kvheads,
                       head_dim=dim)


def test_golden_reference_vectors():
    import kvmem_b200 as K
    golden = json.load(open(GOLDEN))
    scorer = K.PageSoftmaxCuda(0)
    dev = torch.device("cuda", 0)
    for c in golden["page_softmax"]:
        L, P, R, D, Hq, Hkv = c["L"], c["P"], c["R"], c["D"], c["Hq"], c["Hkv"]
        sums = np.frombuffer(base64.b64decode(c["sums_f32_b64"]), np.float32).reshape(L, P, Hkv * D)
        q = np.frombuffer(base64.b64decode(c["q_f32_b64"]), np.float32).reshape(L, R, Hq * D)
        accepted = (P - 1) * c["block"] + c["counts"][-1]
        frame = O.query_score_frame(accepted, c["block"], c["budget"], c["sink"], c["recent"], c["fixed"])
        counts = np.asarray(c["counts"], np.uint32)
        for agg, key in ((0, "expected_mean"), (1, "expected_max")):
            got = scorer.score(torch.from_numpy(sums.copy()).to(dev), torch.from_numpy(counts.view(np.int32)).to(dev),
                               torch.from_numpy(q.copy()).to(dev), c["layer_rows"], frame, agg, q_heads=Hq,
                               kv_heads=Hkv, head_dim=D)
            ok, worst = within(got, c[key])
            assert ok, (agg, worst)


def test_nonfinite_operand_rejected_and_retry_is_identical():
    import kvmem_b200 as K
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    sums = torch.from_numpy(rng.standard_normal((1, 16, 64)).astype(np.float32)).to(dev)
    counts = torch.full((16,), 4, dtype=torch.int32, device=dev)
    q = torch.from_numpy(rng.standard_normal((1, 2, 128)).astype(np.float32)).to(dev)
    frame = O.query_score_frame(64, 4, 32, 0, 0)
    scorer = K.PageSoftmaxCuda(0)
    first = scorer.score(sums, counts, q, [2], frame, 0, q_heads=2, kv_heads=1, head_dim=64)
    bad = q.clone()
    bad[0, 1, 5] = float("nan")
    with pytest.raises(ValueError):
        scorer.score(sums, counts, bad, [2], frame, 0, q_heads=2, kv_heads=1, head_dim=64)
    big = q.clone()
    big[0, 0, 0] = 70000.0  # rounds to FP16 infinity
    with pytest.raises(ValueError):
        scorer.score(sums, counts, big, [2], frame, 0, q_heads=2, kv_heads=1, head_dim=64)
    again = scorer.score(sums, counts, q, [2], frame, 0, q_heads=2, kv_heads=1, head_dim=64)
    assert again == first
