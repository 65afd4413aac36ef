"""GPU: working-set transfers (kvm_transfer), the GPU side of kvmem::MemoryTransfer.

Follows the contract of kvmem/include/kvmem/memory_contract.hpp:171-195 as
kvmem::MemorySession drives it (kvmem/src/host/memory_contract.cpp:245-365):
prepare plans into a shadow (the published view stays intact), spill writes back
evicted pages whose host copy is stale before any slot is reused, restore fills
the new slots, publish exposes the new view, abort drains first and preserves the
previous view only while no restore has started.
"""
import numpy as np
import pytest
import torch

import kvmem_b200 as K

pytestmark = pytest.mark.gpu

ROWS, PAGES, SLOTS, BUDGET, PBYTES = 3, 40, 8, 8, 4096


def _setup(ctx, seed):
    rng = np.random.default_rng(seed)
    host = torch.from_numpy(rng.integers(0, 256, ROWS * PAGES * PBYTES, dtype=np.uint8)).pin_memory()
    cache = torch.zeros(ROWS * SLOTS * PBYTES, dtype=torch.uint8, device="cuda")
    layout = K.stage_layout([dict(host_base=host.data_ptr(), host_row_stride=PAGES * PBYTES, host_page_stride=PBYTES,
                                  dev_base=cache.data_ptr(), dev_row_stride=SLOTS * PBYTES, dev_slot_stride=PBYTES,
                                  bytes=PBYTES)])
    return rng, host, cache, layout


def _select(ctx, rng):
    scores = torch.tensor(rng.random((ROWS, PAGES)).astype(np.float32), device="cuda")
    return ctx.select_topk(scores, [0, PAGES - 1], BUDGET)


def _check_cache(pool, host, cache):
    slot_of, _ = pool.read()
    h = host.numpy().reshape(ROWS, PAGES, PBYTES)
    c = cache.cpu().numpy().reshape(ROWS, SLOTS, PBYTES)
    for r in range(ROWS):
        for p in np.nonzero(slot_of[r] >= 0)[0]:
            assert np.array_equal(c[r, slot_of[r, p]], h[r, p]), (r, p)


def test_transfer_cycle_matches_direct_plan_and_stage(ctx):
    """Three steps through prepare/spill/restore/publish give the same tables and bytes as
    kvm_plan_residency + kvm_stagein_pool on a twin pool."""
    rng, host, cache, layout = _setup(ctx, 0)
    cache2 = torch.zeros_like(cache)
    layout2 = K.stage_layout([dict(host_base=host.data_ptr(), host_row_stride=PAGES * PBYTES,
                                   host_page_stride=PBYTES, dev_base=cache2.data_ptr(),
                                   dev_row_stride=SLOTS * PBYTES, dev_slot_stride=PBYTES, bytes=PBYTES)])
    pool, twin = K.ResidencyPool(ctx, ROWS, PAGES, SLOTS), K.ResidencyPool(ctx, ROWS, PAGES, SLOTS)
    try:
        for step in range(3):
            ids, n = _select(ctx, rng)
            force = step == 2
            t = K.Transfer(pool, ids, n, force_reload=force)
            t.start_spill(layout)
            t.wait()
            t.start_restore(layout, ctas=4)
            t.wait()
            t.publish()
            t.close()
            twin.plan(ids, n, force_reload=force)
            twin.stage_in(layout2, ctas=4)
            torch.cuda.synchronize()
            a, b = pool.read(), twin.read()
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])
            np.testing.assert_array_equal(cache.cpu().numpy(), cache2.cpu().numpy())
            _check_cache(pool, host, cache)
        ctx.check_status("transfer")
    finally:
        pool.close()
        twin.close()


def test_spill_writes_back_stale_evicted_pages(ctx):
    rng, host, cache, layout = _setup(ctx, 1)
    pool = K.ResidencyPool(ctx, ROWS, PAGES, SLOTS)
    try:
        ids, n = _select(ctx, rng)
        t = K.Transfer(pool, ids, n)
        t.start_spill(layout)
        t.wait()
        t.start_restore(layout)
        t.wait()
        t.publish()
        t.close()
        slot_of, _ = pool.read()
        # The device copies of the resident pages change (new KV written on the GPU); every
        # page is marked stale, so the evicted ones must reach their host records.
        cache.add_(1)
        torch.cuda.synchronize()
        dev_before = cache.cpu().numpy().reshape(ROWS, SLOTS, PBYTES).copy()
        host_before = host.numpy().reshape(ROWS, PAGES, PBYTES).copy()
        stale = torch.ones((ROWS, PAGES), dtype=torch.uint8, device="cuda")
        stale[:, 1::2] = 0  # odd pages: host copy current, no write-back
        ids2, n2 = _select(ctx, rng)
        t = K.Transfer(pool, ids2, n2)
        t.start_spill(layout, stale=stale)
        t.wait()
        t.start_restore(layout)
        t.wait()
        t.publish()
        t.close()
        new_slot_of, _ = pool.read()
        h = host.numpy().reshape(ROWS, PAGES, PBYTES)
        for r in range(ROWS):
            for p in np.nonzero(slot_of[r] >= 0)[0]:
                evicted = new_slot_of[r, p] != slot_of[r, p]
                if evicted and p % 2 == 0:
                    assert np.array_equal(h[r, p], dev_before[r, slot_of[r, p]]), (r, p)
                else:
                    assert np.array_equal(h[r, p], host_before[r, p]), (r, p)
        # restored pages hold their host records; retained pages keep the device's newer bytes
        c = cache.cpu().numpy().reshape(ROWS, SLOTS, PBYTES)
        for r in range(ROWS):
            for p in np.nonzero(new_slot_of[r] >= 0)[0]:
                s = new_slot_of[r, p]
                if slot_of[r, p] == s:
                    assert np.array_equal(c[r, s], dev_before[r, s]), (r, p)
                else:
                    assert np.array_equal(c[r, s], h[r, p]), (r, p)
    finally:
        pool.close()


def test_abort_before_restore_preserves_previous_view(ctx):
    rng, host, cache, layout = _setup(ctx, 2)
    pool = K.ResidencyPool(ctx, ROWS, PAGES, SLOTS)
    try:
        ids, n = _select(ctx, rng)
        t = K.Transfer(pool, ids, n)
        t.start_spill(layout)
        t.wait()
        t.start_restore(layout)
        t.wait()
        t.publish()
        t.close()
        before = pool.read()
        cache_before = cache.cpu().numpy().copy()
        ids2, n2 = _select(ctx, rng)
        t = K.Transfer(pool, ids2, n2)
        with pytest.raises(K.KvmError) as e:  # one pending transfer per pool
            K.Transfer(pool, ids2, n2)
        assert e.value.code == K._abi.ERR_PENDING
        with pytest.raises(K.KvmError) as e:  # restore before spill
            t.start_restore(layout)
        assert e.value.code == K._abi.ERR_INVALID_PLAN
        with pytest.raises(K.KvmError) as e:  # publish before restore
            t.publish()
        assert e.value.code == K._abi.ERR_PENDING
        t.start_spill(layout)
        assert t.abort() is True
        after = pool.read()
        np.testing.assert_array_equal(before[0], after[0])
        np.testing.assert_array_equal(before[1], after[1])
        np.testing.assert_array_equal(cache.cpu().numpy(), cache_before)
        with pytest.raises(K.KvmError) as e:
            t.poll()
        assert e.value.code == K._abi.ERR_INVALID_SESSION
        t.close()
        # the pool accepts a new transfer after the abort
        t = K.Transfer(pool, ids2, n2)
        t.start_spill(layout)
        t.wait()
        t.start_restore(layout)
        assert t.abort() is False  # a restore had started: previous view not preserved
        t.close()
    finally:
        pool.close()


def test_abort_that_cannot_drain_keeps_the_pool_blocked(ctx):
    """An abort whose bounded host wait runs out (1 us, while a ~1 GiB restore streams over
    PCIe) reports KVM_ERR_TIMEOUT and keeps the pool blocked: a new prepare is refused
    with KVM_ERR_PENDING until the transfer is destroyed (which drains it), and the
    transfer's own status word, not the context's, decides its publish."""
    rows, pages, slots, pbytes = 8, 64, 32, 4 << 20  # 8 rows x 32 pages x 4 MiB = 1 GiB restored
    host = torch.empty(rows * pages * pbytes, dtype=torch.uint8).pin_memory()
    host.view(-1)[::4096] = 7
    cache = torch.zeros(rows * slots * pbytes, dtype=torch.uint8, device="cuda")
    layout = K.stage_layout([dict(host_base=host.data_ptr(), host_row_stride=pages * pbytes,
                                  host_page_stride=pbytes, dev_base=cache.data_ptr(),
                                  dev_row_stride=slots * pbytes, dev_slot_stride=pbytes, bytes=pbytes)])
    pool = K.ResidencyPool(ctx, rows, pages, slots)
    lib = ctx.lib
    import ctypes as C
    try:
        scores = torch.rand((rows, pages), device="cuda")
        ids, n = ctx.select_topk(scores, [], slots)
        t = K.Transfer(pool, ids, n)
        t.start_spill(layout)
        t.wait()
        t.start_restore(layout, ctas=8)
        kept = C.c_int(1)
        rc = lib.kvm_transfer_abort(t.h, 1, C.byref(kept))
        assert rc == K._abi.ERR_TIMEOUT and kept.value == 0
        with pytest.raises(K.KvmError) as e:
            K.Transfer(pool, ids, n)
        assert e.value.code == K._abi.ERR_PENDING
        assert lib.kvm_transfer_destroy(t.h) == K._abi.OK  # drains, then frees
        t.h = None
        t2 = K.Transfer(pool, ids, n)  # the pool is free again
        t2.abort()
        t2.close()
        # a non-finite score on the context fails that selection's status, not a transfer
        bad = torch.full((1, pages), float("nan"), device="cuda")
        ctx.select_topk(bad, [], 4)
        t3 = K.Transfer(pool, ids, n, force_reload=True)
        t3.start_spill(layout)
        t3.wait()
        t3.start_restore(layout)
        t3.wait()
        t3.publish()
        t3.close()
        assert ctx.status() == K._abi.ERR_NONFINITE  # still there for its owner
    finally:
        torch.cuda.synchronize()
        pool.close()
