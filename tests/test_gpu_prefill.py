"""GPU parity: kvm_prefill_attention (causal prompt attention with the page LSE of sampled rows
captured in the same pass; tcgen05) against the FP64 oracle (oracle.prefill_attention) and against
the separate path (kvm_score_pages over the sampled rows with a causal mask).

Cases: the reference's own capture cases (tests/experimental/prompt_page_lse.cpp qualify() in
backends/patches/ninfer-blackwell-prefill-page-lse.patch:24-31: base / width / sampled rows
(0, 99, {0,31,32,62,63,64,94,98}), (47, 137, 64 rows 2i), (1003, 1024, {5,20,...,1023}) and
(36864, 1024, 32 rows 32i+31), at its admission shape D 256, 24 query / 4 KV heads), in bf16
(the engine's FP8 KV codec is not part of the reference), plus fp16 at D 128 over page sizes 16 to
256, large-logit needles that make rows rescale their accumulator mid-history, key-range splits
merged by the second pass, and argument errors.

Tolerances: attention rows, relative L2 <= 1e-2 (bf16) / 3e-3 (fp16) and max |err| <= 2e-2 of the
row's largest |value| (P and the output are rounded to 16 bits); page LSE within 2e-4 + 1e-5 |lse|
with -inf exactly where the oracle has it; page masses within 1e-5 of the FP64 masses and of the
separate path's."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def make(seed, base, width, hq, hkv, dim, dtype, needles=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    T = base + width
    q = torch.randn(width, hq, dim, generator=g)
    k = torch.randn(T, hkv, dim, generator=g)
    v = torch.randn(T, hkv, dim, generator=g)
    if needles:
        # Keys aligned with late prompt rows' queries: their logits jump by ~|q|^2 * scale, so those rows
        # raise their running max far past the lazy-rescale threshold mid-history.
        rows = torch.randint(width // 2, width, (needles,), generator=g)
        for r in rows.tolist():
            h = int(torch.randint(0, hq, (1,), generator=g))
            t = int(torch.randint(base // 2, base + r + 1, (1,), generator=g))
            k[t, h // (hq // hkv)] = q[r, h] * 1.5
    q, k, v = (x.to(dtype) for x in (q, k, v))
    return q, k, v


def check_rows(got, exp, dtype):
    rel = 1e-2 if dtype == torch.bfloat16 else 3e-3
    for i in range(exp.shape[0]):
        e, o = exp[i], got[i].astype(np.float64)
        err = np.linalg.norm(o - e) / max(np.linalg.norm(e), 1e-30)
        assert err <= rel, f"row {i}: relative L2 {err:.3g}"
        assert np.abs(o - e).max() <= 2e-2 * max(1.0, np.abs(e).max())


def check_lse(got, exp):
    inf_e, inf_g = ~np.isfinite(exp), ~np.isfinite(got)
    assert (inf_e == inf_g).all(), f"{int((inf_e != inf_g).sum())} -inf mismatches"
    assert (got[inf_g] == -np.inf).all()
    d = np.abs(got[~inf_g] - exp[~inf_e])
    tol = 2e-4 + 1e-5 * np.abs(exp[~inf_e])
    assert (d <= tol).all(), f"page LSE: worst {d.max():.3g}, {int((d > tol).sum())} out of tolerance"


def run(ctx, *, base, width, samples, hq=24, hkv=4, dim=256, dtype=torch.bfloat16, pt=64, check=None, needles=0,
        seed=0, pages=None):
    q, k, v = make(seed, base, width, hq, hkv, dim, dtype, needles)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out, lse = ctx.prefill_attention(qd, kd, vd, base=base, sample_rows=samples, page_tokens=pt, pages=pages)
    torch.cuda.synchronize()
    ctx.check_status("prefill_attention")
    check = sorted(set(check if check is not None else range(width)) | set(samples))
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    exp_o, exp_l = O.prefill_attention(qn, kn, vn, base=base, rows=check, sample_rows=samples, page_tokens=pt,
                                       pages=pages or 0)
    check_rows(out.float().cpu().numpy()[check], exp_o, dtype)
    if samples:
        got_l = lse.cpu().numpy()
        check_lse(got_l, exp_l)
        return qd, kd, vd, got_l, exp_l
    assert lse is None
    return qd, kd, vd, None, None


@pytest.mark.parametrize("base,width,samples", [
    (0, 99, [0, 31, 32, 62, 63, 64, 94, 98]),
    (47, 137, [2 * i for i in range(64)]),
    (1003, 1024, [5, 20, 63, 85, 196, 511, 751, 1023]),
])
def test_reference_capture_cases(ctx, base, width, samples):
    check = None if width <= 137 else list(range(0, width, 37)) + [width - 1]
    *_, got_l, exp_l = run(ctx, base=base, width=width, samples=samples, check=check)
    desc = ctx.make_desc(layers=1, q_heads=24, kv_heads=4, head_dim=256, tokens=got_l.shape[2] * 64, page_tokens=64)
    mass, _ = ctx.page_mass_from_lse(desc, len(samples), torch.from_numpy(got_l).to(DEV), want_mean=False)
    np.testing.assert_allclose(mass.cpu().numpy()[0, 0], O.page_mass_from_lse(exp_l), atol=1e-5, rtol=0)


def test_long_history_capture_equals_separate_statistics(ctx):
    """The reference's long case (base 36864, width 1024, 32 sampled rows): the fused capture's page
    masses equal both the FP64 masses and the separate path's (kvm_score_pages over the sampled rows,
    causal visibility as a -inf bias)."""
    import kvmem_b200 as K
    base, width, hq, hkv, dim = 36864, 1024, 24, 4, 256
    samples = [32 * i + 31 for i in range(32)]
    qd, kd, vd, got_l, exp_l = run(ctx, base=base, width=width, samples=samples, check=samples[::8], needles=8)
    T = base + width
    pages = got_l.shape[2]
    desc = ctx.make_desc(layers=1, q_heads=hq, kv_heads=hkv, head_dim=dim, tokens=T, page_tokens=64)
    fused, _ = ctx.page_mass_from_lse(desc, len(samples), torch.from_numpy(got_l).to(DEV), want_mean=False)
    np.testing.assert_allclose(fused.cpu().numpy()[0, 0], O.page_mass_from_lse(exp_l), atol=1e-5, rtol=0)
    qs = qd[samples].contiguous().view(1, len(samples), hq, dim)
    pos = torch.tensor([base + r for r in samples], device=DEV)
    mask = torch.where(torch.arange(T, device=DEV)[None, :] <= pos[:, None], 0.0, float("-inf")).float()
    sdesc = K.RecallContext.make_desc(layers=1, q_heads=hq, kv_heads=hkv, head_dim=dim, tokens=T, page_tokens=64,
                                      mask=mask)
    sq = K.RecallContext.make_query(qs, len(samples))
    sk = K.RecallContext.make_kcache(kd, K.BF16, kv_heads=hkv, head_dim=dim, capacity_tokens=T)
    sep, _ = ctx.score_pages(sdesc, sq, sk, want_mean=False)
    torch.cuda.synchronize()
    ctx.check_status("score_pages")
    assert sep.shape[-1] == pages
    np.testing.assert_allclose(fused.cpu().numpy(), sep.cpu().numpy(), atol=1e-5, rtol=0)


@pytest.mark.parametrize("pt", [16, 32, 64, 128, 256])
def test_fp16_d128_page_sizes(ctx, pt):
    base, width = 300, 200
    samples = [0, 1, 63, 64, 127, 128, 150, 199]
    run(ctx, base=base, width=width, samples=samples, hq=8, hkv=2, dim=128, dtype=torch.float16, pt=pt, needles=4,
        seed=pt, pages=-(-(base + width) // pt) + 3)


def test_bf16_d128_and_fp16_d256(ctx):
    run(ctx, base=129, width=257, samples=[3, 128, 255, 256], hq=16, hkv=4, dim=128, dtype=torch.bfloat16, needles=3)
    run(ctx, base=64, width=130, samples=[129], hq=8, hkv=8, dim=256, dtype=torch.float16, pt=128, needles=3)


def test_attention_only_and_single_row(ctx):
    run(ctx, base=500, width=77, samples=[], hq=8, hkv=2, dim=128, dtype=torch.bfloat16)
    run(ctx, base=0, width=1, samples=[0], hq=4, hkv=1, dim=256, dtype=torch.bfloat16)


@pytest.mark.parametrize("splits", [2, 3, 5])
def test_key_range_split_merge(ctx, monkeypatch, splits):
    """Each row tile's keys cut into chunks merged by the second pass (forced with
    KVM_PREFILL_SPLITS): chunks of whole 256-token capture pages, empty trailing chunks and
    rows that see no key of a chunk (base 0) all give the unsplit result."""
    monkeypatch.setenv("KVM_PREFILL_SPLITS", str(splits))
    run(ctx, base=1003, width=300, samples=[5, 20, 63, 85, 196, 299], check=list(range(0, 300, 13)), needles=6)
    run(ctx, base=700, width=150, samples=[0, 77, 149], hq=8, hkv=2, dim=128, dtype=torch.float16, pt=256,
        needles=3, seed=splits)
    run(ctx, base=0, width=260, samples=[0, 1, 200], hq=8, hkv=2, dim=128, dtype=torch.bfloat16, pt=32)


def test_more_samples_than_the_first_capture_took(ctx):
    """Every row of a 260-row chunk sampled (the dynamic-sample capture, rows from device memory),
    then a second call with a different list: each matches the oracle."""
    run(ctx, base=300, width=260, samples=list(range(260)), hq=8, hkv=2, dim=128, dtype=torch.bfloat16,
        check=[0, 100, 259])
    run(ctx, base=41, width=200, samples=list(range(1, 200, 3)), hq=8, hkv=2, dim=128, dtype=torch.float16,
        check=[1, 199], seed=5)


def test_argument_errors(ctx):
    import kvmem_b200 as K
    q, k, v = (x.to(DEV) for x in make(1, 64, 64, 8, 2, 128, torch.bfloat16))
    with pytest.raises(K.KvmError):  # unsorted sample rows
        ctx.prefill_attention(q, k, v, base=64, sample_rows=[5, 3])
    with pytest.raises(K.KvmError):  # a sample past the prompt
        ctx.prefill_attention(q, k, v, base=64, sample_rows=[64])
    with pytest.raises(K.KvmError):  # too few capture columns
        ctx.prefill_attention(q, k, v, base=64, sample_rows=[1], pages=1)
    with pytest.raises(K.KvmError):  # a page size the capture does not take
        ctx.prefill_attention(q, k, v, base=64, sample_rows=[1], page_tokens=48)
    with pytest.raises(K.KvmError):  # the cache holds fewer keys than base + width
        ctx.prefill_attention(q, k[:100], v[:100], base=64, sample_rows=[1])
    with pytest.raises(K.KvmError):  # a repeated sample row
        ctx.prefill_attention(q, k, v, base=64, sample_rows=list(range(64)) + [63])
    with pytest.raises(K.KvmError):  # head_dim 64 is not served
        q64, k64, v64 = (x.to(DEV) for x in make(1, 64, 64, 8, 2, 64, torch.bfloat16))
        ctx.prefill_attention(q64, k64, v64, base=64)
    torch.cuda.synchronize()
    ctx.check_status("after rejected calls")
