"""GPU: stage-out of device page bytes into the double-buffered pinned slots.

Follows the reference's reverse slab (src/adapter/llama-kvmem-stagein.cu:883-1004)
and its caller's batching (harvest_gpu_v / harvest_gpu_v_flush_slab,
src/adapter/llama-memory-kvmem.cpp:3935-4050): regions are queued with their
slot offsets, a full batch is submitted into the current slot while the host
consumes the previous one, and every staged byte must equal the device bytes.
"""
import numpy as np
import pytest
import torch

import kvmem_b200 as K

pytestmark = pytest.mark.gpu


def _device_bytes(rng, n):
    return torch.from_numpy(rng.integers(0, 256, n, dtype=np.uint8)).cuda()


def test_random_regions_byte_exact():
    rng = np.random.default_rng(1)
    src = _device_bytes(rng, 8 << 20)
    host = src.cpu().numpy()
    so = K.StageOut(0, slot_bytes=4 << 20, max_items=64)
    try:
        for rnd in range(3):
            items = []
            while True:
                n = int(rng.integers(1, 300_000))
                start = int(rng.integers(0, src.numel() - n))
                if rnd == 0:
                    start &= ~15  # aligned sources in the first round, any byte offset afterwards
                off = so.enqueue(src.data_ptr() + start, n)
                if off is None:
                    break
                assert off % 16 == 0
                items.append((start, n, off))
            assert items
            slot = so.submit(ctas=int(rng.integers(1, 40)))
            assert slot == rnd % 2
            so.wait(slot)
            for start, n, off in items:
                np.testing.assert_array_equal(so.slot_view(slot, off, n), host[start:start + n])
    finally:
        so.close()


def test_harvest_double_buffer_sequence():
    """K and V rows of every layer of filled blocks, batched like the reference's harvest."""
    rng = np.random.default_rng(2)
    layers, slots, block_rows, row_k, row_v = 8, 6, 256, 272, 144  # q8_0 K / q4_0 V, 4 heads x 256 dims
    k_cache = _device_bytes(rng, layers * slots * block_rows * row_k)
    v_cache = _device_bytes(rng, layers * slots * block_rows * row_v)
    kh, vh = k_cache.cpu().numpy(), v_cache.cpu().numpy()
    so = K.StageOut(0, slot_bytes=1 << 20, max_items=16)
    got = {}

    def consume(batch):
        slot, jobs = batch
        if slot < 0:
            return
        so.wait(slot)
        for key, off, n in jobs:
            got[key] = so.slot_view(slot, off, n).copy()

    pending, jobs = (-1, []), []
    try:
        for gpu_slot in (4, 1, 5, 0):
            n_tok = int(rng.integers(1, block_rows + 1))
            for il in range(layers):
                for is_k, cache, row in ((True, k_cache, row_k), (False, v_cache, row_v)):
                    nbytes = n_tok * row
                    base = (il * slots + gpu_slot) * block_rows * row
                    key = (gpu_slot, il, is_k, base, nbytes)
                    off = so.used()
                    if so.enqueue(cache.data_ptr() + base, nbytes) is None:
                        # flush: finish the pending batch, submit this one, continue in the other slot
                        slot = so.submit()
                        consume(pending)
                        pending, jobs = (slot, jobs), []
                        off = so.used()
                        assert so.enqueue(cache.data_ptr() + base, nbytes) == off
                    jobs.append((key, off, nbytes))
        slot = so.submit()
        consume(pending)
        consume((slot, jobs))
    finally:
        so.close()
    assert len(got) == 4 * layers * 2
    for (gpu_slot, il, is_k, base, nbytes), data in got.items():
        ref = kh if is_k else vh
        np.testing.assert_array_equal(data, ref[base:base + nbytes])


def test_edge_cases():
    src = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    so = K.StageOut(0, slot_bytes=1 << 16, max_items=2)
    try:
        assert so.submit() == -1  # nothing queued
        so.wait(-1)
        assert so.enqueue(src.data_ptr(), (1 << 16) + 16) is None  # larger than a slot
        assert so.enqueue(src.data_ptr(), 100) == 0
        assert so.used() == 112
        assert so.enqueue(src.data_ptr() + 7, 9) == 112
        assert so.enqueue(src.data_ptr(), 1) is None  # max_items reached
        so.clear()
        assert so.used() == 0 and so.submit() == -1
        with pytest.raises(K.KvmError) as e:
            so.enqueue(0, 16)
        assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
        with pytest.raises(K.KvmError):
            so.wait(2)
    finally:
        so.close()
    with pytest.raises(K.KvmError):
        K.StageOut(0, slot_bytes=100)  # not a multiple of 16
