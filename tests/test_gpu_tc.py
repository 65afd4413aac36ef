"""GPU parity of the tcgen05 page scorer (query replay / multi-lane batching).

The tcgen05 kernel scores 16 or more query vectors per KV head (rows x group)
against fp16 keys with head_dim 64, 128 or 256: up to 160 vectors per launch
(128 at head_dim 256), more in equal passes. Every case runs twice: with
KVM_SCORER=tc, which makes kvm_score_pages fail unless that kernel runs, and
with KVM_SCORER=mma (the mma.sync kernel) on the same inputs; both are compared
with the FP64 oracle at the north-star tolerance of 1e-3 relative.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import util as U
from tests.test_gpu_page_mass import ABS, REL, run_case

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["tc", "mma"])
def scorer(request, monkeypatch):
    monkeypatch.setenv("KVM_SCORER", request.param)
    return request.param


CASES = [
    # config-4 shape, reduced history: 32 replay rows x 40/8 heads -> 160 vectors per KV head (two M tiles)
    dict(ktype=U.F16, D=128, Hq=40, Hkv=8, R=32, page=128, T=1024, L=2),
    # one M tile: 4 rows x 5 heads
    dict(ktype=U.F16, D=128, Hq=40, Hkv=8, R=4, page=128, T=1024),
    # M-tile edges: 128, 129, 144 and 160 vectors
    dict(ktype=U.F16, D=128, Hq=8, Hkv=2, R=32, page=64, T=512),
    dict(ktype=U.F16, D=64, Hq=43, Hkv=1, R=3, page=64, T=256),
    dict(ktype=U.F16, D=64, Hq=16, Hkv=2, R=18, page=32, T=320),
    dict(ktype=U.F16, D=64, Hq=10, Hkv=2, R=32, page=64, T=700, L=2),
    # head_dim 64, pages of 32, partial last page, spare capacity, three layers
    dict(ktype=U.F16, D=64, Hq=16, Hkv=4, R=8, page=32, T=1000, cap=1088, L=3),
    # pages of 256 and 384 tokens (several tiles per page)
    dict(ktype=U.F16, D=128, Hq=24, Hkv=4, R=4, page=256, T=2048),
    dict(ktype=U.F16, D=128, Hq=12, Hkv=2, R=3, page=384, T=1500),
    # per-KV-head aggregation groups, f16 and bf16 queries, explicit scale, softcap
    dict(ktype=U.F16, D=128, Hq=32, Hkv=8, R=8, page=64, T=512, groups=8),
    dict(ktype=U.F16, D=128, Hq=40, Hkv=8, R=4, page=128, T=640, qtype=U.F16),
    dict(ktype=U.F16, D=64, Hq=40, Hkv=8, R=8, page=128, T=640, qtype=U.BF16, scale=0.2),
    dict(ktype=U.F16, D=128, Hq=16, Hkv=4, R=8, page=64, T=512, softcap=30.0, scale=0.25),
    # f16 queries on the 129..160-vector layout (the tile-0 lo MMAs are skipped: every lo part is 0)
    dict(ktype=U.F16, D=128, Hq=40, Hkv=8, R=32, page=128, T=512, L=2, qtype=U.F16),
    dict(ktype=U.F16, D=64, Hq=40, Hkv=8, R=30, page=64, T=384, qtype=U.BF16),
    # head_dim 256 (config-2 / 3 / 5 heads, sampled rows): 24 and 126 vectors in one launch
    dict(ktype=U.F16, D=256, Hq=24, Hkv=4, R=4, page=256, T=2048),
    dict(ktype=U.F16, D=256, Hq=24, Hkv=4, R=21, page=256, T=1100, L=2),
    # several passes: 160 vectors at head_dim 256 (2 x 80), 384 (3 x 128), 200 at head_dim 128
    # (2 x 100) and 256 at head_dim 64 (2 x 128)
    dict(ktype=U.F16, D=256, Hq=16, Hkv=2, R=20, page=128, T=700, L=2),
    dict(ktype=U.F16, D=256, Hq=24, Hkv=4, R=64, page=256, T=1024),
    dict(ktype=U.F16, D=128, Hq=40, Hkv=8, R=40, page=128, T=640),
    dict(ktype=U.F16, D=64, Hq=16, Hkv=2, R=32, page=32, T=320),
    # head_dim 256 with f16 queries and a softcap
    dict(ktype=U.F16, D=256, Hq=24, Hkv=4, R=8, page=256, T=1024, qtype=U.F16, softcap=20.0, scale=0.1),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
def test_tc_page_mass_matches_oracle(ctx, scorer, case):
    got, exp = run_case(ctx, **case)
    np.testing.assert_allclose(got.sum(axis=-1), 1.0, atol=2e-5)


@pytest.mark.parametrize("mag", [1e-4, 1.0, 3e3])
def test_tc_query_magnitudes(ctx, scorer, mag):
    """Queries far from unit scale: the per-vector power-of-two prescale keeps the
    fp16 hi / lo split exact enough at both ends (scale adjusted so logits stay O(1))."""
    import kvmem_b200 as K
    rng = np.random.default_rng(11)
    L, R, Hq, Hkv, D, T, page = 1, 8, 16, 4, 128, 512, 64
    kb = U.make_k(rng, U.F16, L, T, Hkv, D)
    qf = (rng.standard_normal((L, R, Hq, D)) * mag).astype(np.float32)
    scale = float(np.float32(1.0 / (np.sqrt(D) * mag)))
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qf).to(dev)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page,
                                     scale=scale)
    rows, _ = ctx.score_pages(desc, K.RecallContext.make_query(q_d, R),
                              K.RecallContext.make_kcache(k_d, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=T),
                              want_mean=False)
    torch.cuda.synchronize()
    ctx.check_status("score_pages")
    exp = O.page_mass(qf.view(np.uint8), U.F32, kb, U.F16, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D,
                      tokens=T, page_tokens=page, scale=scale)
    ok, worst, nbad = U.close(rows.cpu().numpy(), exp, REL, ABS)
    assert ok, f"worst {worst:.3g}, {nbad} pages"


@pytest.mark.parametrize("D", [128, 256])
def test_tc_mask_and_empty_rows(ctx, scorer, D):
    """Additive mask rows on the tcgen05 path: hidden tokens, a causal tail, a
    bias row, and a fully hidden row whose masses are NaN as the reference's."""
    import kvmem_b200 as K
    rng = np.random.default_rng(5)
    L, R, Hq, Hkv, T, page = 1, 8, 16, 4, 640, 128
    mask = np.zeros((R, T), np.float32)
    mask[0, 100:300] = -np.inf
    mask[1, :] = rng.standard_normal(T).astype(np.float32)
    mask[2, :] = -np.inf
    for r in range(3, R):
        mask[r, 500 + 10 * r:] = -np.inf
    kb = U.make_k(rng, U.F16, L, T, Hkv, D)
    qb = U.make_q(rng, U.F32, L, R, Hq, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, R, Hq, D)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page,
                                     mask=torch.from_numpy(mask).to(dev))
    rows, _ = ctx.score_pages(desc, K.RecallContext.make_query(q_d, R),
                              K.RecallContext.make_kcache(k_d, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=T),
                              want_mean=False)
    torch.cuda.synchronize()
    got = rows.cpu().numpy()
    exp = O.page_mass(qb, U.F32, kb, U.F16, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=page, scale=1 / np.sqrt(D), mask=mask)
    assert np.isnan(got[0, 0, 2]).all() and np.isnan(exp[0, 0, 2]).all()
    keep = [r for r in range(R) if r != 2]
    ok, worst, _ = U.close(got[:, :, keep], exp[:, :, keep], REL, ABS)
    assert ok, worst


@pytest.mark.parametrize("rows,page", [(1, 64), (32, 96)])
def test_tc_strict_mode_rejects_other_shapes(ctx, monkeypatch, rows, page):
    """KVM_SCORER=tc refuses shapes outside the tcgen05 kernel: 8 vectors per KV head
    (fewer than 16), and pages of 96 tokens (neither a divisor nor a multiple of 128)."""
    import kvmem_b200 as K
    monkeypatch.setenv("KVM_SCORER", "tc")
    dev = torch.device("cuda", 0)
    k_d = torch.zeros(288 * 2 * 128 * 2, dtype=torch.uint8, device=dev)
    q_d = torch.zeros((1, rows, 16, 128), dtype=torch.float32, device=dev)
    desc = K.RecallContext.make_desc(layers=1, q_heads=16, kv_heads=2, head_dim=128, tokens=288, page_tokens=page)
    with pytest.raises(K.KvmError) as e:
        ctx.score_pages(desc, K.RecallContext.make_query(q_d, rows),
                        K.RecallContext.make_kcache(k_d, U.F16, kv_heads=2, head_dim=128, capacity_tokens=288))
    assert e.value.code == K._abi.ERR_UNSUPPORTED


def test_default_scorer_takes_tc_passes_for_large_batches(ctx, monkeypatch):
    """384 vectors per KV head at head_dim 256 under the default scorer choice: three
    tcgen05 passes (3 launches of the LSE kernel + the normaliser), still exact."""
    monkeypatch.setenv("KVM_SCORER", "auto")
    before = ctx.launches
    run_case(ctx, ktype=U.F16, D=256, Hq=24, Hkv=4, R=64, page=256, T=768)
    assert ctx.launches - before == 4


@pytest.mark.parametrize("case", [dict(D=128, Hq=40, Hkv=8, R=32, page=128, T=1024, L=2),
                                  dict(D=128, Hq=40, Hkv=8, R=4, page=128, T=700, L=1),
                                  dict(D=64, Hq=16, Hkv=4, R=8, page=64, T=1000, L=3, cap=1088),
                                  dict(D=128, Hq=24, Hkv=4, R=4, page=256, T=2048, L=2),
                                  dict(D=256, Hq=24, Hkv=4, R=8, page=256, T=2048, L=2)],
                         ids=["160v", "20v_partial", "d64_3layers", "page256", "d256"])
def test_head_major_mirror_matches_oracle(ctx, case):
    """A head-major K score mirror ([layer][kv_head][token][D]: each head's rows contiguous)
    scored by the tcgen05 kernel equals the FP64 oracle on the token-major bytes; the other
    scorers reject that layout (KVM_ERR_UNSUPPORTED)."""
    import kvmem_b200 as K
    from kvmem_b200 import _abi as A
    D, Hq, Hkv, R, page, T, L = (case[k] for k in ("D", "Hq", "Hkv", "R", "page", "T", "L"))
    cap = case.get("cap", -(-T // page) * page)
    rng = np.random.default_rng(D + R + L)
    kb = U.make_k(rng, U.F16, L, cap, Hkv, D)  # token-major bytes [L][cap][Hkv][row]
    qb = U.make_q(rng, U.F32, L, R, Hq, D)
    dev = torch.device("cuda", 0)
    rb = U.row_bytes(U.F16, D)
    mirror = torch.from_numpy(np.ascontiguousarray(kb.transpose(0, 2, 1, 3)).reshape(-1)).to(dev)
    kc = A.KCache()
    kc.data, kc.type = mirror.data_ptr(), U.F16
    kc.token_stride, kc.head_stride, kc.layer_stride = rb, cap * rb, Hkv * cap * rb
    kc.capacity_tokens = cap
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, R, Hq, D)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page)
    rows, _ = ctx.score_pages(desc, K.RecallContext.make_query(q_d, R), kc, want_mean=False)
    torch.cuda.synchronize()
    ctx.check_status("head-major")
    scale = float(np.float32(1) / np.sqrt(np.float32(D)))
    exp = O.page_mass(qb, U.F32, kb, U.F16, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=page, scale=scale, k_strides=(cap * Hkv * rb, Hkv * rb, rb))
    ok, worst, nbad = U.close(rows.cpu().numpy(), exp, REL, ABS)
    assert ok, f"{nbad} pages off, worst {worst:.3g}"
    one = K.RecallContext.make_query(q_d, 1, strides=(R * Hq * D * 4, Hq * D * 4, D * 4))  # too few vectors
    with pytest.raises(K.KvmError) as e:
        ctx.score_pages(desc, one, kc, want_mean=False)
    assert e.value.code == A.ERR_UNSUPPORTED
