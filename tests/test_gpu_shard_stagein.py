"""GPU: stage-in of a page-range partition (kvm_shard_stagein) equals the whole stage-in.

The ranks of a page-range partition keep identical residency tables (each plans the
same merged selection) and each gathers only the restores of its own page range from
its own range's records. Emulated here on one GPU: three "ranks", each with its own
pool copy and its own slice of the host records, write into one cache; after every
step the cache, and every pool copy's tables, must equal a single pool's plan and
whole-range stage-in (kvm_plan_residency + kvm_stagein_pool) byte for byte.
"""
import numpy as np
import pytest
import torch

import kvmem_b200 as K
from kvmem_b200.shard import page_ranges

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ranks", [1, 3])
def test_range_stagein_equals_whole(ctx, ranks):
    rows, pages, slots, kbytes, vbytes = 4, 45, 9, 8192, 2304
    rng = np.random.default_rng(ranks)
    hk = rng.integers(0, 256, (rows, pages, kbytes), dtype=np.uint8)
    hv = rng.integers(0, 256, (rows, pages, vbytes), dtype=np.uint8)
    host_k = torch.from_numpy(hk.reshape(-1).copy()).pin_memory()
    host_v = torch.from_numpy(hv.reshape(-1).copy()).pin_memory()
    whole_k = torch.zeros(rows * slots * kbytes, dtype=torch.uint8, device="cuda")
    whole_v = torch.zeros(rows * slots * vbytes, dtype=torch.uint8, device="cuda")
    part_k, part_v = torch.zeros_like(whole_k), torch.zeros_like(whole_v)

    def layout(hbase_k, hbase_v, row_pages, dk, dv):
        return K.stage_layout([
            dict(host_base=hbase_k, host_row_stride=row_pages * kbytes, host_page_stride=kbytes,
                 dev_base=dk.data_ptr(), dev_row_stride=slots * kbytes, dev_slot_stride=kbytes, bytes=kbytes),
            dict(host_base=hbase_v, host_row_stride=row_pages * vbytes, host_page_stride=vbytes,
                 dev_base=dv.data_ptr(), dev_row_stride=slots * vbytes, dev_slot_stride=vbytes, bytes=vbytes)])

    whole = K.ResidencyPool(ctx, rows, pages, slots)
    whole_layout = layout(host_k.data_ptr(), host_v.data_ptr(), pages, whole_k, whole_v)
    parts = []
    for p0, p1 in page_ranges(pages, ranks):
        rk = torch.from_numpy(np.ascontiguousarray(hk[:, p0:p1]).reshape(-1)).pin_memory()
        rv = torch.from_numpy(np.ascontiguousarray(hv[:, p0:p1]).reshape(-1)).pin_memory()
        parts.append((p0, p1, K.ResidencyPool(ctx, rows, pages, slots),
                      layout(rk.data_ptr(), rv.data_ptr(), p1 - p0, part_k, part_v), rk, rv))
    try:
        for step in range(6):
            scores = torch.tensor(rng.random((rows, pages)).astype(np.float32), device="cuda")
            ids, n = ctx.select_topk(scores, [0, pages - 1], slots)
            force = step == 4
            whole.plan(ids, n, force_reload=force)
            whole.stage_in(whole_layout)
            for p0, p1, pool, lay, _, _ in parts:
                pool.plan(ids, n, force_reload=force)
                pool.stage_in_range(lay, p0, p1 - p0, ctas=3)
            torch.cuda.synchronize()
            ctx.check_status(f"step {step}")
            want = whole.read()
            for _, _, pool, _, _, _ in parts:
                got = pool.read()
                np.testing.assert_array_equal(got[0], want[0])
                np.testing.assert_array_equal(got[1], want[1])
            assert torch.equal(part_k, whole_k) and torch.equal(part_v, whole_v), f"step {step}"
            # and the cache holds the host records of the resident pages
            slot_of = want[0]
            ck = whole_k.cpu().numpy().reshape(rows, slots, kbytes)
            for r in range(rows):
                for p in np.nonzero(slot_of[r] >= 0)[0]:
                    assert np.array_equal(ck[r, slot_of[r, p]], hk[r, p])
        with pytest.raises(K.KvmError):  # a range past the pool's pages is rejected
            parts[0][2].stage_in_range(parts[0][3], pages - 1, 2)
    finally:
        whole.close()
        for part in parts:
            part[2].close()
