"""Generates tests/golden/reference_cases.json from the reference's own CPU code.

Runs the reference library compiled from its sources (oracle/_ref/libkvref.so,
``make -C oracle ref``) on seeded inputs and records inputs and outputs of
  query_score_frame   (kvmem/src/host/graph_recall.cpp:269)
  recall_fp16         (kvmem/src/host/graph_recall.cpp:295)
  page_softmax_scores (kvmem/src/host/graph_recall.cpp:322), Mean and Max
  pick_scored_blocks  (kvmem/src/host/kvmem_store.cpp:418)
  plan_residency      (kvmem/src/host/memory_contract.cpp:135)
The fixtures pin the C restatement in oracle/ and, through it, the GPU kernels.
Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import base64
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_cases.json")


def frames():
    cases = []
    for args in [(12, 4, 2, 0, 0, [2]), (11, 4, 4, 1, 1, [0, 2]), (12, 4, 2, 1, 1, [0, 2]), (1000, 64, 8, 1, 2, [3]),
                 (16384, 64, 16, 1, 1, [0, 255]), (131072, 256, 34, 1, 1, []), (300, 128, 1, 0, 0, [])]:
        f = O.query_score_frame(*args, use_ref=True)
        cases.append(dict(args=list(args[:5]), fixed=args[5], score_mask=f["score_mask"].tolist(),
                          transport_mask=f["transport_mask"].tolist(), counts=f["counts"].tolist()))
    return cases


def recall():
    vals = [1.00048828125, 1.00146484375, 2.0 ** -24, 2.0 ** -25, 1.5 * 2.0 ** -25, 65504.0, 65519.0, 65520.0,
            65536.0, -3.14159, 1e-8, -6.1e-5, 6.2e-5, 0.0, -0.0, 1234.5678, float("inf"), float("nan")]
    rng = np.random.default_rng(1)
    vals += [float(x) for x in rng.standard_normal(32).astype(np.float32) * 100]
    out = []
    for v in vals:
        try:
            out.append([repr(v), O.recall_fp16(v, use_ref=True)])
        except ValueError:
            out.append([repr(v), None])
    return out


def page_softmax():
    cases = []
    rng = np.random.default_rng(7)
    shapes = [  # (layers, pages, rows, dim, heads, kv_heads, block, budget, sink, recent, fixed)
        (2, 7, 3, 64, 8, 2, 4, 3, 1, 1, [0, 6]),
        (1, 40, 2, 32, 4, 1, 16, 8, 1, 2, []),
        (3, 17, 1, 128, 6, 2, 8, 20, 0, 0, []),
        (2, 64, 4, 64, 4, 4, 32, 10, 2, 1, [5]),
    ]
    for (L, P, R, D, Hq, Hkv, block, budget, sink, recent, fixed) in shapes:
        expected = []
        for agg in (0, 1):
            kw = Hkv * D
            counts = np.full(P, block, np.uint32)
            counts[-1] = max(1, block // 2 + 1)
            sums = (rng.standard_normal((L, P, kw)).astype(np.float32) * counts[None, :, None] * 0.5).astype(np.float32)
            q = rng.standard_normal((L, R, Hq * D)).astype(np.float32)
            layer_rows = np.full(L, R, np.uint32)
            if L > 2:
                layer_rows[1] = 0  # an absent layer
            accepted = int((P - 1) * block + counts[-1])
            if agg == 1:  # same operands for both aggregations
                sums, q = sums0, q0
            sums0, q0 = sums, q
            out = O.ref_page_softmax_scores(sums, counts, q, layer_rows, heads=Hq, kv_heads=Hkv, dim=D, block=block,
                                            accepted=accepted, budget=budget, sink=sink, recent=recent, fixed=fixed,
                                            aggregation=agg)
            expected.append(out.tolist())
        cases.append(dict(L=L, P=P, R=R, D=D, Hq=Hq, Hkv=Hkv, block=block, budget=budget, sink=sink,
                          recent=recent, fixed=fixed, counts=counts.tolist(),
                          sums_f32_b64=base64.b64encode(sums.tobytes()).decode(),
                          q_f32_b64=base64.b64encode(q.tobytes()).decode(),
                          layer_rows=layer_rows.tolist(), expected_mean=expected[0], expected_max=expected[1]))
    return cases


def pick():
    cases = []
    rng = np.random.default_rng(11)
    for i in range(24):
        n = int(rng.integers(4, 300))
        scores = rng.random(n)
        if i % 3 == 0:  # many exact ties
            scores = np.round(scores * 4) / 4
        if i % 5 == 0:
            scores[rng.integers(0, n, 5)] = 0.0
        signed = i % 4 == 3
        if signed:
            scores = scores - 0.5
        scores = scores.astype(np.float32).astype(np.float64)  # the GPU ranks f32 scores
        budget = int(rng.integers(1, n + 3))
        nm = int(rng.integers(0, min(4, budget) + 1))
        mandatory = sorted(set(int(x) for x in rng.integers(0, n, nm)))
        if i % 6 == 1:
            mandatory = [0, n - 1][: min(2, budget)]
        rc, ids = O.pick_scored(n, list(range(n)), scores, mandatory, budget, signed=signed, use_ref=True)
        cases.append(dict(n=n, scores=scores.tolist(), mandatory=mandatory, budget=budget, signed=signed, rc=rc,
                          ids=None if ids is None else ids.tolist()))
    # rejected inputs: negative unsigned score, mandatory over budget
    cases.append(dict(n=4, scores=[0.1, -0.2, 0.3, 0.4], mandatory=[], budget=2, signed=False,
                      rc=O.pick_scored(4, [0, 1, 2, 3], [0.1, -0.2, 0.3, 0.4], [], 2, use_ref=True)[0], ids=None))
    cases.append(dict(n=5, scores=[0.1] * 5, mandatory=[0, 1, 2], budget=2, signed=False,
                      rc=O.pick_scored(5, list(range(5)), [0.1] * 5, [0, 1, 2], 2, use_ref=True)[0], ids=None))
    return cases


def media_pick():
    # graph_recall_test.cpp:242-253 fixture shape (blocks of 4 tokens, two media ranges).
    out = []
    for cand, scores, mand, budget in [([0, 1, 2, 3, 4, 5], [0, 0, 0, 0, 9, 8], [0, 3], 4),
                                       ([0, 3, 4, 5], [0, 1, 9, 8], [0, 3], 4),
                                       ([0, 1, 2, 3, 4, 5], [5, 4, 3, 2, 1, 0], [], 3)]:
        rc, ids = O.pick_scored(6, cand, scores, mand, budget, block_tokens=4, ranges=[(4, 9), (9, 13)],
                                use_ref=True)
        out.append(dict(cand=cand, scores=scores, mandatory=mand, budget=budget, rc=rc,
                        ids=None if ids is None else ids.tolist()))
    return out


def residency():
    cases = []
    rng = np.random.default_rng(5)
    for i in range(16):
        universe = int(rng.integers(5, 200))
        res = sorted(set(int(x) for x in rng.integers(0, universe, int(rng.integers(0, 30)))))
        sel = sorted(set(int(x) for x in rng.integers(0, universe, int(rng.integers(0, 30)))))
        force = i % 4 == 0
        rc, d = O.plan_residency(res, sel, force, use_ref=True)
        cases.append(dict(resident=res, selected=sel, force=force, rc=rc,
                          evict=d["evict"].tolist(), retain=d["retain"].tolist(), restore=d["restore"].tolist()))
    rc, _ = O.plan_residency([1, 1], [2], False, use_ref=True)
    cases.append(dict(resident=[1, 1], selected=[2], force=False, rc=rc, evict=None, retain=None, restore=None))
    return cases


def main():
    O.build(ref=True)
    if O.ref() is None:
        raise SystemExit("reference library unavailable (needs the reference sources)")
    data = dict(frames=frames(), recall_fp16=recall(), page_softmax=page_softmax(), pick=pick(),
                media_pick=media_pick(), residency=residency())
    with open(OUT, "w") as f:
        json.dump(data, f)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
