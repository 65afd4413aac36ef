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


def test_noalloc_mask_and_replay_batch_against_oracle():
    """A replay-shaped batch (4 rows x 5 query heads per KV head: the tcgen05 scorer) with an
    additive mask (a causal tail per row and a hidden span), through the no-allocation entry
    point, checked against the FP64 oracle as well as against kvm_score_pages."""
    import kvmem_b200 as K
    from oracle import oracle as O
    lib = K._abi.load()
    rng = np.random.default_rng(21)
    L, R, Hq, Hkv, D, T, page = 2, 4, 40, 8, 128, 1024, 128
    mask = np.zeros((R, T), np.float32)
    mask[0, 200:400] = -np.inf
    for r in range(1, R):
        mask[r, T - 60 * r:] = -np.inf
    kb = U.make_k(rng, U.F16, L, T, Hkv, D)
    qb = U.make_q(rng, U.F32, L, R, Hq, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, R, Hq, D)
    m_d = torch.from_numpy(mask).to(dev)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page,
                                     mask=m_d)
    q = K.RecallContext.make_query(q_d, R)
    k = K.RecallContext.make_kcache(k_d, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=T)
    P = T // page
    got_rows = torch.full((L, 1, R, P), float("nan"), device="cuda")
    rc = lib.kvm_score_pages_noalloc(C.byref(desc), C.byref(q), C.byref(k), got_rows.data_ptr(), None,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == K._abi.OK, K._abi.STATUS_NAMES.get(rc)
    torch.cuda.synchronize()
    exp = O.page_mass(qb, U.F32, kb, U.F16, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=page, scale=float(np.float32(1) / np.sqrt(np.float32(D))), mask=mask)
    ok, worst, _ = U.close(got_rows.cpu().numpy(), exp, REL, ABS)
    assert ok, f"noalloc masses differ from the FP64 oracle (worst {worst:.3g})"
    ctx = K.RecallContext(0)
    want_rows, _ = ctx.score_pages(desc, q, k, want_mean=False)
    torch.cuda.synchronize()
    ok, worst, _ = U.close(got_rows.cpu().numpy(), want_rows.cpu().numpy(), REL, ABS)
    assert ok, f"noalloc masses differ from kvm_score_pages (worst {worst:.3g})"
    ctx.close()
