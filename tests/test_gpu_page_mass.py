"""GPU parity: kvm_score_pages (per-token page mass) against the FP64 oracle.

Tolerance (fp32 accumulation vs FP64): |gpu - oracle| <= 1e-6 + 1e-3 * |oracle|
per page mass, the north-star bound of 1e-3 relative on page scores.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import util as U

pytestmark = pytest.mark.gpu

REL, ABS = 1e-3, 1e-6
QT = {U.F32: torch.float32, U.F16: torch.float16, U.BF16: torch.bfloat16}


@pytest.fixture(params=["auto", "simt", "mma_generic"])
def scorer(request, monkeypatch):
    """Every page scorer: the tensor-core kernels (auto, where they apply), the FP32 SIMT kernel,
    and the fp16 mma.sync kernel for quantised keys (mma_generic)."""
    monkeypatch.setenv("KVM_SCORER", request.param)
    return request.param


def run_case(ctx, *, ktype, D, Hq, Hkv, R=1, L=2, page=64, T=1024, cap=None, groups=1, qtype=U.F32, softcap=0.0,
             mask=None, scale=0.0, seed=0):
    import kvmem_b200 as K
    rng = np.random.default_rng(seed)
    cap = cap or -(-T // page) * page
    kb = U.make_k(rng, ktype, L, cap, Hkv, D)
    qb = U.make_q(rng, qtype, L, R, Hq, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(QT[qtype]).view(L, R, Hq, D)
    mask_d = None
    if mask is not None:
        mask_d = torch.from_numpy(mask).to(dev)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page,
                                     groups=groups, scale=scale, softcap=softcap, mask=mask_d)
    q = K.RecallContext.make_query(q_d, R)
    k = K.RecallContext.make_kcache(k_d, ktype, kv_heads=Hkv, head_dim=D, capacity_tokens=cap)
    rows, mean = ctx.score_pages(desc, q, k)
    torch.cuda.synchronize()
    ctx.check_status("score_pages")
    eff_scale = scale if scale > 0 else float(np.float32(1.0) / np.sqrt(np.float32(D)))
    exp = O.page_mass(qb, qtype, kb, ktype, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=page, scale=eff_scale, softcap=softcap, groups=groups,
                      mask=mask, k_strides=(cap * Hkv * U.row_bytes(ktype, D), Hkv * U.row_bytes(ktype, D),
                                            U.row_bytes(ktype, D)))
    got = rows.cpu().numpy()
    ok, worst, nbad = U.close(got, exp, REL, ABS)
    assert ok, f"mass_rows differs from the FP64 oracle: worst {worst:.3g}, {nbad} pages out of tolerance"
    ok, worst, nbad = U.close(mean.cpu().numpy(), exp.mean(axis=2), REL, ABS)
    assert ok, f"mass_mean differs: worst {worst:.3g}"
    return got, exp


CASES = [
    # config-1 shape, reduced history: D128, 32/8 heads, page 64
    dict(ktype=U.F16, D=128, Hq=32, Hkv=8, page=64, T=1024),
    # config-2 shape, reduced: D256, 24/4 heads (G=6), page 256
    dict(ktype=U.F16, D=256, Hq=24, Hkv=4, page=256, T=2048, L=2),
    # config-3 encodings: q8_0 keys, D256, 24/4
    dict(ktype=U.Q8_0, D=256, Hq=24, Hkv=4, page=256, T=1024),
    dict(ktype=U.Q8_0, D=128, Hq=8, Hkv=2, page=64, T=512),
    dict(ktype=U.Q4_0, D=128, Hq=8, Hkv=2, page=64, T=512),
    dict(ktype=U.Q4_0, D=256, Hq=8, Hkv=1, page=32, T=300),
    dict(ktype=U.Q5_0, D=64, Hq=4, Hkv=4, page=16, T=256),
    dict(ktype=U.BF16, D=128, Hq=16, Hkv=4, page=32, T=512, qtype=U.BF16),
    dict(ktype=U.F32, D=64, Hq=8, Hkv=8, page=16, T=200, qtype=U.F16),
    # config-4 shape, reduced: replay rows R=4, 40/8 heads (G=5) -> 20 query vectors per KV head
    dict(ktype=U.F16, D=128, Hq=40, Hkv=8, R=4, page=128, T=1024),
    # partial last page and spare capacity
    dict(ktype=U.F16, D=128, Hq=8, Hkv=2, page=64, T=1000, cap=1088),
    # per-KV-head aggregation groups
    dict(ktype=U.F16, D=128, Hq=32, Hkv=8, page=64, T=512, groups=8),
    dict(ktype=U.Q8_0, D=256, Hq=24, Hkv=4, page=256, T=768, groups=4, R=2),
    # softcap and explicit scale
    dict(ktype=U.F16, D=256, Hq=8, Hkv=4, page=64, T=512, softcap=30.0, scale=0.25),
    # f16 queries (no lo part), MQA (one KV head), large query magnitudes (prescale)
    dict(ktype=U.F16, D=64, Hq=8, Hkv=1, page=64, T=512, qtype=U.F16),
    dict(ktype=U.Q4_0, D=256, Hq=24, Hkv=4, page=256, T=768, qtype=U.BF16),
    dict(ktype=U.Q8_0, D=128, Hq=40, Hkv=8, R=2, page=128, T=512),
    # quantised keys across the quantised kernel's variants: head_dim 64 (two blocks),
    # 8 and 1 KV heads, partial last page, softcap, f16 queries
    dict(ktype=U.Q8_0, D=64, Hq=16, Hkv=8, page=64, T=512),
    dict(ktype=U.Q4_0, D=64, Hq=4, Hkv=2, page=128, T=1000, cap=1024),
    dict(ktype=U.Q8_0, D=256, Hq=24, Hkv=4, page=256, T=700, cap=768, softcap=30.0),
    dict(ktype=U.Q8_0, D=128, Hq=8, Hkv=1, page=64, T=512, qtype=U.F16),
    dict(ktype=U.Q4_0, D=128, Hq=16, Hkv=8, page=64, T=640, softcap=20.0, scale=0.1),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
def test_page_mass_matches_oracle(ctx, scorer, case):
    got, exp = run_case(ctx, **case)
    # each (layer, group, row) distribution sums to 1
    np.testing.assert_allclose(got.sum(axis=-1), 1.0, atol=2e-5)


def test_mask_hides_tokens_and_empty_rows_are_nan(ctx, scorer):
    R, T = 3, 512
    mask = np.zeros((R, T), np.float32)
    mask[0, 100:300] = -np.inf
    mask[1, :] = np.random.default_rng(1).standard_normal(T).astype(np.float32)
    mask[2, :] = -np.inf  # nothing visible: NaN, as the reference's normaliser yields
    import kvmem_b200 as K
    rng = np.random.default_rng(4)
    D, Hq, Hkv, page, L = 128, 8, 2, 64, 1
    kb = U.make_k(rng, U.F16, L, T, Hkv, D)
    qb = U.make_q(rng, U.F32, L, R, Hq, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, R, Hq, D)
    m_d = torch.from_numpy(mask).to(dev)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page,
                                     mask=m_d)
    rows, _ = ctx.score_pages(desc, K.RecallContext.make_query(q_d, R),
                              K.RecallContext.make_kcache(k_d, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=T),
                              want_mean=False)
    torch.cuda.synchronize()
    got = rows.cpu().numpy()
    exp = O.page_mass(qb, U.F32, kb, U.F16, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=page, scale=1 / np.sqrt(D), mask=mask)
    assert np.isnan(got[0, 0, 2]).all() and np.isnan(exp[0, 0, 2]).all()
    ok, worst, _ = U.close(got[:, :, :2], exp[:, :, :2], REL, ABS)
    assert ok, worst
    assert got[0, 0, 0, 2] < 1e-6  # page 2 (tokens 128..191) fully hidden for row 0


@pytest.mark.parametrize("ktype", [U.Q8_0, U.Q4_0])
def test_quantised_keys_with_mask(ctx, scorer, ktype):
    R, T, page = 2, 640, 64
    rng = np.random.default_rng(7)
    mask = rng.standard_normal((R, T)).astype(np.float32)
    mask[0, 64:200] = -np.inf
    mask[1, 600:] = -np.inf
    run_case(ctx, ktype=ktype, D=256, Hq=24, Hkv=4, R=R, page=page, T=T, mask=mask, seed=3)


@pytest.mark.parametrize("ktype", [U.Q8_0, U.Q4_0])
def test_quantised_keys_with_outlier_queries(ctx, scorer, ktype):
    """Query channels 30x / 100x the rest, vectors scaled by 1e-3 and 30, and all-zero blocks:
    the quantised-key scorer splits each 32-element query block into two int8 digits under
    the block's own power of two, so small elements next to an outlier keep 2^-15 of the
    outlier's magnitude; page masses must still meet the 1e-3 relative bound."""
    import kvmem_b200 as K
    rng = np.random.default_rng(11)
    L, R, Hq, Hkv, D, T, page = 2, 2, 24, 4, 256, 1024, 256
    q = rng.standard_normal((L, R, Hq, D)).astype(np.float32)
    q[..., [5, 77, 200]] *= 30.0
    q[..., 130] *= 100.0
    q[:, 0, 0] *= 1e-3
    q[:, 1, 1] *= 30.0
    q[:, :, 2, 32:64] = 0.0  # one block of zeros
    qb = U.encode(q, U.F32).reshape(L, R, Hq, -1)
    kb = U.make_k(rng, ktype, L, T, Hkv, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(q.copy()).to(dev)
    desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T, page_tokens=page)
    rows, _ = ctx.score_pages(desc, K.RecallContext.make_query(q_d, R),
                              K.RecallContext.make_kcache(k_d, ktype, kv_heads=Hkv, head_dim=D, capacity_tokens=T))
    torch.cuda.synchronize()
    ctx.check_status("score_pages")
    exp = O.page_mass(qb, U.F32, kb, ktype, layers=L, rows=R, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=page, scale=float(np.float32(1.0) / np.sqrt(np.float32(D))))
    ok, worst, nbad = U.close(rows.cpu().numpy(), exp, REL, ABS)
    assert ok, f"worst {worst:.3g}, {nbad} pages out of tolerance"


def test_unsupported_layouts_are_rejected(ctx):
    import kvmem_b200 as K
    dev = torch.device("cuda", 0)
    k_d = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    q_d = torch.zeros((1, 1, 8, 96), dtype=torch.float32, device=dev)
    desc = K.RecallContext.make_desc(layers=1, q_heads=8, kv_heads=2, head_dim=96, tokens=256, page_tokens=64)
    with pytest.raises(K.KvmError) as e:  # head_dim 96 is outside the kernel's set
        ctx.score_pages(desc, K.RecallContext.make_query(q_d, 1),
                        K.RecallContext.make_kcache(k_d, U.F16, kv_heads=2, head_dim=96, capacity_tokens=256))
    assert e.value.code == K._abi.ERR_UNSUPPORTED
    q_d = torch.zeros((1, 1, 8, 128), dtype=torch.float32, device=dev)
    desc = K.RecallContext.make_desc(layers=1, q_heads=8, kv_heads=2, head_dim=128, tokens=300, page_tokens=64)
    with pytest.raises(K.KvmError) as e:  # last page not allocated
        ctx.score_pages(desc, K.RecallContext.make_query(q_d, 1),
                        K.RecallContext.make_kcache(k_d, U.F16, kv_heads=2, head_dim=128, capacity_tokens=300))
    assert e.value.code == K._abi.ERR_UNSUPPORTED
    desc = K.RecallContext.make_desc(layers=1, q_heads=6, kv_heads=4, head_dim=128, tokens=256, page_tokens=64)
    with pytest.raises(K.KvmError) as e:  # heads not a multiple of kv heads
        ctx.score_pages(desc, K.RecallContext.make_query(q_d, 1),
                        K.RecallContext.make_kcache(k_d, U.F16, kv_heads=4, head_dim=128, capacity_tokens=256))
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT


def test_attention_cuda_mirror_matches_oracle(scorer):
    """The llama_kvmem_attention_cuda mirror: ggml-style views, sampled rows, mask rows."""
    import kvmem_b200 as K
    rng = np.random.default_rng(9)
    D, Hq, Hkv, T, block, nrows = 128, 16, 4, 512, 64, 40
    kb = U.make_k(rng, U.Q8_0, 1, T, Hkv, D)
    qb = U.make_q(rng, U.F32, 1, nrows, Hq, D)
    mask = np.zeros((nrows, T), np.float32)
    for r in range(nrows):
        mask[r, 400 + r:] = -np.inf  # causal tail
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev)
    m_d = torch.from_numpy(mask).to(dev)
    rb = U.row_bytes(U.Q8_0, D)
    qv = K.TensorView(q_d, U.F32, (D, nrows, Hq), (4, Hq * D * 4, D * 4))
    kv = K.TensorView(k_d, U.Q8_0, (D, T, Hkv), (1, Hkv * rb, rb))
    mv = K.TensorView(m_d, U.F32, (T, nrows, 1), (4, T * 4, 0))
    sampler = K.AttentionCuda(0)
    rows = [3, 17, 39]
    out = sampler.score(qv, kv, mv, 1 / np.sqrt(D), 0.0, block, rows)
    assert out is not None and len(out) == 3
    exp = O.page_mass(qb, U.F32, kb, U.Q8_0, layers=1, rows=nrows, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                      page_tokens=block, scale=1 / np.sqrt(D), mask=mask)
    for i, r in enumerate(rows):
        ok, worst, _ = U.close(out[i], exp[0, 0, r], REL, ABS)
        assert ok, worst
    # head_dim beyond 256 is outside the kernel: the reference returns false
    big = K.TensorView(q_d, U.F32, (288, 1, 1), (4, 288 * 4, 288 * 4))
    assert sampler.score(big, kv, mv, 1.0, 0.0, block, [0]) is None
