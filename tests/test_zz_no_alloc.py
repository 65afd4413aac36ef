"""GPU test of kvm_score_pages_noalloc, the page-mass entry point that allocates nothing.

Callers that cannot allocate device memory while scoring (an engine whose
device memory is all claimed up front by its own pool, a plugin host that
forbids new allocations after start-up) call this variant; its scratch is a
fixed array reserved by the driver when the library loads. This test calls it
through the C ABI twice in a row, on different inputs, and checks each result
against kvm_score_pages (the allocating entry point) with the tolerance of the
other page-mass tests. It lives in its own file, collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from tests import util as U

pytestmark = pytest.mark.gpu
REL, ABS = 1e-3, 1e-6


def inputs(seed, ktype):
    import kvmem_b200 as K
    rng = np.random.default_rng(seed)
    L, Hq, Hkv, D, T, page = 4, 24, 4, 256, 4096, 256
    kb = U.make_k(rng, ktype, L, T, Hkv, D)
    qb = U.make_q(rng, U.F32, L, 1, Hq, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, 1, Hq, D)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T - 100,
                                     page_tokens=page)
    q = K.RecallContext.make_query(q_d, 1)
    k = K.RecallContext.make_kcache(k_d, ktype, kv_heads=Hkv, head_dim=D, capacity_tokens=T)
    return desc, q, k, (k_d, q_d), (L, T // page)


def test_noalloc_matches_allocating_entry_point_twice():
    import kvmem_b200 as K
    lib = K._abi.load()
    ctx = K.RecallContext(0)
    stream = torch.cuda.current_stream().cuda_stream
    for seed, ktype in ((11, U.F16), (12, U.Q8_0)):
        desc, q, k, keep_alive, (L, P) = inputs(seed, ktype)
        want_rows, want_mean = ctx.score_pages(desc, q, k)
        got_rows = torch.full((L, 1, 1, P), float("nan"), device="cuda")
        got_mean = torch.full((L, 1, P), float("nan"), device="cuda")
        rc = lib.kvm_score_pages_noalloc(C.byref(desc), C.byref(q), C.byref(k), got_rows.data_ptr(),
                                         got_mean.data_ptr(), stream)
        assert rc == K._abi.OK, K._abi.STATUS_NAMES.get(rc)
        torch.cuda.synchronize()
        ok, worst, _ = U.close(got_rows.cpu().numpy(), want_rows.cpu().numpy(), REL, ABS)
        assert ok, f"noalloc rows differ from kvm_score_pages (worst {worst:.3g})"
        ok, worst, _ = U.close(got_mean.cpu().numpy(), want_mean.cpu().numpy(), REL, ABS)
        assert ok, f"noalloc means differ from kvm_score_pages (worst {worst:.3g})"
    ctx.close()


def test_noalloc_rejects_problems_beyond_its_scratch():
    import kvmem_b200 as K
    lib = K._abi.load()
    desc, q, k, keep_alive, _ = inputs(13, U.F16)
    # 64 layers x 24 heads x 2048 pages x 4 B = 12.6 MB of page LSE > 8 MiB. The call
    # returns before any launch, so the small K buffer is never read.
    desc.layers, desc.tokens = 64, 2048 * 256
    k.capacity_tokens = 2048 * 256
    k.layer_stride = 2048 * 256 * k.token_stride
    rc = lib.kvm_score_pages_noalloc(C.byref(desc), C.byref(q), C.byref(k), None, None,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == K._abi.ERR_LENGTH
