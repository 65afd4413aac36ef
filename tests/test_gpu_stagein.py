"""GPU parity: device residency plan against plan_residency, and byte-exact stage-in.

The device pool follows plan_residency (kvmem/src/host/memory_contract.cpp:135-150)
for the sets; restored pages take freed slots in ascending page / slot order.
The staged cache bytes must equal the host page bytes exactly.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


class SlotModel:
    """Host model of the pool: the oracle's residency delta + the ascending slot rule."""

    def __init__(self, rows, pages, slots):
        self.slot_of = -np.ones((rows, pages), np.int32)
        self.page_of = -np.ones((rows, slots), np.int32)

    def apply(self, r, selected, force):
        resident = [int(p) for p in np.nonzero(self.slot_of[r] >= 0)[0]]
        rc, d = O.plan_residency(resident, selected, force)
        assert rc == 0
        for p in d["evict"]:
            s = self.slot_of[r, p]
            self.slot_of[r, p] = -1
            self.page_of[r, s] = -1
        free = [int(s) for s in np.nonzero(self.page_of[r] < 0)[0]]
        for p, s in zip(d["restore"], free):
            self.slot_of[r, p] = s
            self.page_of[r, s] = p
        return d


def test_plan_sequence_matches_oracle(ctx):
    import kvmem_b200 as K
    rows, pages, slots, budget = 4, 60, 10, 10
    pool = K.ResidencyPool(ctx, rows, pages, slots)
    model = SlotModel(rows, pages, slots)
    rng = np.random.default_rng(0)
    for step in range(12):
        force = step == 7
        scores = torch.tensor(rng.random((rows, pages)).astype(np.float32), device="cuda")
        ids, n = ctx.select_topk(scores, [0, pages - 1], budget)
        n_restore, n_evict = pool.plan(ids, n, force_reload=force)
        torch.cuda.synchronize()
        assert ctx.status() == 0
        ids_h, n_h = ids.cpu().numpy(), n.cpu().numpy()
        for r in range(rows):
            d = model.apply(r, ids_h[r, : n_h[r]].tolist(), force)
            assert int(n_restore[r]) == len(d["restore"])
            assert int(n_evict[r]) == len(d["evict"])
        slot_of, page_of = pool.read()
        np.testing.assert_array_equal(slot_of, model.slot_of)
        np.testing.assert_array_equal(page_of, model.page_of)


@pytest.mark.parametrize("kbytes,vbytes", [(2048, 1024), (4352, 2304), (1000, 36)])
def test_stagein_bytes_exact(ctx, kbytes, vbytes):
    """K and V page records from pinned host memory land byte-exact in their slots
    (4352/2304 = one q8_0 / q4_0 page of 16 tokens x D256; 1000/36 = unaligned byte path)."""
    import kvmem_b200 as K
    rows, pages, slots, budget = 3, 40, 6, 6
    rng = np.random.default_rng(kbytes)
    host_k = torch.from_numpy(rng.integers(0, 256, rows * pages * kbytes, dtype=np.uint8)).pin_memory()
    host_v = torch.from_numpy(rng.integers(0, 256, rows * pages * vbytes, dtype=np.uint8)).pin_memory()
    dev_k = torch.zeros(rows * slots * kbytes, dtype=torch.uint8, device="cuda")
    dev_v = torch.zeros(rows * slots * vbytes, dtype=torch.uint8, device="cuda")
    layout = K.stage_layout([
        dict(host_base=host_k.data_ptr(), host_row_stride=pages * kbytes, host_page_stride=kbytes,
             dev_base=dev_k.data_ptr(), dev_row_stride=slots * kbytes, dev_slot_stride=kbytes, bytes=kbytes),
        dict(host_base=host_v.data_ptr(), host_row_stride=pages * vbytes, host_page_stride=vbytes,
             dev_base=dev_v.data_ptr(), dev_row_stride=slots * vbytes, dev_slot_stride=vbytes, bytes=vbytes)])
    pool = K.ResidencyPool(ctx, rows, pages, slots)
    hk = host_k.numpy().reshape(rows, pages, kbytes)
    hv = host_v.numpy().reshape(rows, pages, vbytes)
    for step in range(5):
        scores = torch.tensor(rng.random((rows, pages)).astype(np.float32), device="cuda")
        ids, n = ctx.select_topk(scores, [0], budget)
        pool.plan(ids, n, force_reload=(step == 3))
        pool.stage_in(layout, ctas=8)
        ctx.wait(30.0)
        slot_of, _ = pool.read()
        dk = dev_k.cpu().numpy().reshape(rows, slots, kbytes)
        dv = dev_v.cpu().numpy().reshape(rows, slots, vbytes)
        ids_h, n_h = ids.cpu().numpy(), n.cpu().numpy()
        for r in range(rows):
            for p in ids_h[r, : n_h[r]]:
                s = slot_of[r, p]
                assert s >= 0
                assert np.array_equal(dk[r, s], hk[r, p]), (step, r, p)
                assert np.array_equal(dv[r, s], hv[r, p]), (step, r, p)


def test_copy_list(ctx):
    rng = np.random.default_rng(1)
    src = torch.from_numpy(rng.integers(0, 256, 1 << 20, dtype=np.uint8)).pin_memory()
    dst = torch.zeros((1 << 20) + 4096, dtype=torch.uint8, device="cuda")
    ops = [(src.data_ptr() + 4096 * i, dst.data_ptr() + 4096 * (255 - i), 4096) for i in range(256)]
    ops.append((src.data_ptr() + 3, dst.data_ptr() + (1 << 20) + 5, 17))  # unaligned
    ctx.stagein_copies(ops, ctas=16)
    ctx.wait(30.0)
    s, d = src.numpy(), dst.cpu().numpy()
    for i in range(0, 256, 17):
        assert np.array_equal(d[4096 * (255 - i): 4096 * (256 - i)], s[4096 * i: 4096 * (i + 1)])
    assert np.array_equal(d[(1 << 20) + 5:(1 << 20) + 22], s[3:20])


def test_copy_lists_back_to_back(ctx):
    """Several lists enqueued without waiting (the two op lists are reused in turn), of growing
    length, each list's host array dropped as soon as the call returns."""
    rng = np.random.default_rng(2)
    src = torch.from_numpy(rng.integers(0, 256, 8 << 20, dtype=np.uint8)).pin_memory()
    dst = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    expect = np.zeros(8 << 20, np.uint8)
    s = src.numpy()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for call in range(6):
            n = 64 * (call + 1)  # the third list outgrows the first allocation
            chunk = (8 << 20) // (6 * 384)
            base = call * 384 * chunk
            ops = []
            for i in range(n):
                so = int(rng.integers(0, (8 << 20) - chunk))
                do = base + i * chunk
                ops.append((src.data_ptr() + so, dst.data_ptr() + do, chunk))
                expect[do:do + chunk] = s[so:so + chunk]
            ctx.stagein_copies(ops, ctas=8, stream=stream)
    ctx.wait(30.0, stream=stream)
    np.testing.assert_array_equal(dst.cpu().numpy(), expect)
