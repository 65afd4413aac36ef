"""CPU: the library's host-code frame and keep-set builders (no GPU needed) against the
reference's own code: kvm_query_score_frame vs query_score_frame
(kvmem/src/host/graph_recall.cpp:269-293) on the golden frames and random arguments, and
kvm_query_fixed_blocks vs KvMemStore::query_fixed_blocks (kvmem/src/host/kvmem_store.cpp:
381-405) on random stores, both run through the compiled reference (oracle/_ref/libkvref.so)
when it is present, rejections included."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")


def lib_frame(accepted, block, budget, sink, recent, fixed, capacity=None):
    from kvmem_b200 import _abi as A
    L = A.load()
    cap = capacity if capacity is not None else accepted // max(block, 1) + 2
    starts = np.zeros(max(cap, 1), np.uint64)
    counts = np.zeros(max(cap, 1), np.uint32)
    sm = np.zeros(max(cap, 1), np.uint8)
    tm = np.zeros(max(cap, 1), np.uint8)
    fx = (C.c_uint32 * max(1, len(fixed)))(*fixed)
    n = C.c_uint64()
    rc = L.kvm_query_score_frame(accepted, block, budget, sink, recent, fx, len(fixed), cap,
                                 starts.ctypes.data, counts.ctypes.data, sm.ctypes.data, tm.ctypes.data,
                                 C.byref(n))
    k = n.value
    return rc, dict(starts=starts[:k], counts=counts[:k], score_mask=sm[:k], transport_mask=tm[:k])


def test_golden_frames():
    golden = json.load(open(GOLDEN))
    for c in golden["frames"]:
        rc, f = lib_frame(*c["args"], c["fixed"])
        assert rc == 0
        assert f["score_mask"].tolist() == c["score_mask"]
        assert f["transport_mask"].tolist() == c["transport_mask"]
        assert f["counts"].tolist() == c["counts"]
        assert f["starts"].tolist() == [i * c["args"][1] for i in range(len(c["counts"]))]


def test_random_frames_match_reference():
    if O.ref() is None:
        pytest.skip("the compiled reference is absent (reference sources not present at build)")
    rng = np.random.default_rng(4)
    for _ in range(400):
        block = int(rng.integers(1, 300))
        accepted = int(rng.integers(0, 40 * block))
        budget = int(rng.integers(1, 50))
        sink, recent = int(rng.integers(0, 5)), int(rng.integers(0, 5))
        n = -(-accepted // block)
        fixed = sorted(set(int(x) for x in rng.integers(0, n + 2, int(rng.integers(0, 4))))) if n else []
        try:
            want = O.query_score_frame(accepted, block, budget, sink, recent, fixed, use_ref=True)
        except ValueError:
            want = None
        rc, got = lib_frame(accepted, block, budget, sink, recent, fixed)
        if want is None:
            assert rc != 0
            continue
        assert rc == 0
        for key in ("starts", "counts", "score_mask", "transport_mask"):
            assert got[key].tolist() == want[key].tolist(), key


def test_rejections():
    from kvmem_b200 import _abi as A
    assert lib_frame(100, 0, 4, 1, 1, [])[0] == A.ERR_INVALID_ARGUMENT  # no block size
    assert lib_frame(100, 10, 0, 1, 1, [])[0] == A.ERR_INVALID_ARGUMENT  # no budget
    assert lib_frame(100, 10, 4, 1, 1, [10])[0] == A.ERR_INVALID_ARGUMENT  # fixed page outside the index
    assert lib_frame(100, 10, 4, 1, 1, [], capacity=9)[0] == A.ERR_LENGTH  # 10 pages, room for 9


def lib_fixed(total, block, budget, sink, recent, ranges, mandatory):
    from kvmem_b200 import _abi as A
    L = A.load()
    flat = [int(x) for r in ranges for x in r]
    rg = (C.c_uint32 * max(1, len(flat)))(*flat)
    md = (C.c_uint32 * max(1, len(mandatory)))(*mandatory)
    cap = total // block + 2
    out = (C.c_uint32 * cap)()
    n = C.c_uint32()
    rc = L.kvm_query_fixed_blocks(total, block, budget, sink, recent, rg, len(ranges), md, len(mandatory), out, cap,
                                  C.byref(n))
    return rc, list(out[: n.value]) if rc == 0 else None


def ref_fixed(total, block, budget, sink, recent, ranges, mandatory):
    flat = np.ascontiguousarray([int(x) for r in ranges for x in r] or [0], np.uint32)
    md = np.ascontiguousarray(list(mandatory) or [0], np.uint32)
    out = np.zeros(total // block + 2, np.uint32)
    n = C.c_uint32()
    u = C.c_uint32
    rc = O.ref().kvref_query_fixed_blocks(u(total), u(block), u(budget), u(sink), u(recent), C.c_void_p(flat.ctypes.data),
                                          u(len(ranges)), C.c_void_p(md.ctypes.data), u(len(mandatory)),
                                          C.c_void_p(out.ctypes.data), C.byref(n))
    return rc, out[: n.value].tolist() if rc == 0 else None


def test_fixed_blocks_match_reference():
    """kvm_query_fixed_blocks against the compiled reference's KvMemStore::query_fixed_blocks
    (sink, newest media item, mandatory, recent; media groups; budget overflows)."""
    from kvmem_b200 import _abi as A
    if O.ref() is None:
        pytest.skip("the compiled reference is absent (reference sources not present at build)")
    rng = np.random.default_rng(9)
    for it in range(500):
        block = int(rng.integers(1, 64))
        total = int(rng.integers(1, 60 * block))
        n = -(-total // block)
        budget = int(rng.integers(0, 40))
        sink, recent = int(rng.integers(0, 4)), int(rng.integers(0, 6))
        ranges = []
        for _ in range(int(rng.integers(0, 6))):
            a = int(rng.integers(0, total + 2 * block))
            ranges.append((a, a + int(rng.integers(0, 5 * block))))
        mandatory = [int(x) for x in rng.integers(0, n + (1 if it % 7 == 0 else 0), int(rng.integers(0, 4)))]
        rc_ref, want = ref_fixed(total, block, budget, sink, recent, ranges, mandatory)
        rc, got = lib_fixed(total, block, budget, sink, recent, ranges, mandatory)
        if rc_ref == 1:
            assert rc == A.ERR_INVALID_ARGUMENT, (it, rc)
        elif rc_ref == 2:
            assert rc == A.ERR_BUDGET_EXCEEDED, (it, rc)
        else:
            assert rc == 0 and got == want, (it, got, want)
