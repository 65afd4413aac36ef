"""GPU parity: kvm_meank_add (Mean-K producer: per-page K sums kept in HBM).

The device table must equal the oracle's sequential f32 accumulation bit for
bit (restating the reference's meank_add kernels, src/adapter/llama-kvmem-stagein.cu:270-316),
through prefill-sized adds that cross pages and one-token decode adds, for
every key type; the table then feeds kvm_meank_score directly and scores as
the oracle does on means formed from its own sums.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import util as U
from tests.test_gpu_meank import means_from_sums, within

pytestmark = pytest.mark.gpu

ADDS = ((0, 100), (100, 1), (101, 1), (102, 37), (139, 1), (140, 160))  # prefill, decode, a chunk, decode, rest


@pytest.mark.parametrize("kt", [U.F32, U.F16, U.BF16, U.Q8_0, U.Q4_0, U.Q5_0])
@pytest.mark.parametrize("D,Hkv,B", [(128, 4, 64), (64, 2, 32)])
def test_meank_add_bit_exact(ctx, kt, D, Hkv, B):
    import kvmem_b200 as K
    rng = np.random.default_rng(3 + kt)
    L, T = 3, 300
    P = -(-T // B)
    kb = U.make_k(rng, kt, L, T, Hkv, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    kc = K.RecallContext.make_kcache(k_d, kt, kv_heads=Hkv, head_dim=D, capacity_tokens=T)
    sums_d = torch.zeros((L, P, Hkv * D), dtype=torch.float32, device=dev)
    counts_d = torch.zeros((P,), dtype=torch.int32, device=dev)
    sums = np.zeros((L, P, Hkv * D), np.float32)
    counts = np.zeros(P, np.uint32)
    for tok0, n in ADDS:
        ctx.meank_add(kc, sums_d, counts_d, tok0=tok0, n=n, page_tokens=B, kv_heads=Hkv, head_dim=D)
        assert O.meank_add(sums, counts, kb, kt, layers=L, kv_heads=Hkv, dim=D, tok0=tok0, n=n, page_tokens=B) == 0
    torch.cuda.synchronize()
    ctx.check_status("meank_add")
    got = sums_d.cpu().numpy()
    assert np.array_equal(got, sums), f"max |diff| {np.abs(got - sums).max()}"
    assert counts_d.cpu().numpy().astype(np.uint32).tolist() == counts.tolist()


@pytest.mark.parametrize("agg", [0, 1])
def test_produced_table_feeds_meank_score(ctx, agg):
    import kvmem_b200 as K
    rng = np.random.default_rng(17)
    L, T, Hkv, Hq, D, B, R = 2, 640, 4, 16, 128, 64, 3
    P = T // B
    kb = U.make_k(rng, U.F16, L, T, Hkv, D)
    dev = torch.device("cuda", 0)
    k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
    kc = K.RecallContext.make_kcache(k_d, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=T)
    sums_d = torch.zeros((L, P, Hkv * D), dtype=torch.float32, device=dev)
    counts_d = torch.zeros((P,), dtype=torch.int32, device=dev)
    sums = np.zeros((L, P, Hkv * D), np.float32)
    counts = np.zeros(P, np.uint32)
    for tok0 in range(0, T, 80):  # chunks that do not align with pages
        ctx.meank_add(kc, sums_d, counts_d, tok0=tok0, n=80, page_tokens=B, kv_heads=Hkv, head_dim=D)
        O.meank_add(sums, counts, kb, U.F16, layers=L, kv_heads=Hkv, dim=D, tok0=tok0, n=80, page_tokens=B)
    q = (rng.standard_normal((L, R, Hq * D)) * 0.5).astype(np.float32)
    q_d = torch.from_numpy(q).to(dev)
    mask = [1] * P
    mask[0] = mask[-1] = 0  # sink / recent pages outside the denominator
    out = ctx.meank_score(sums_d, counts_d, q_d, [R] * L, mask, q_heads=Hq, kv_heads=Hkv, head_dim=D,
                          aggregation=agg, scale=float(1 / np.sqrt(D)))
    torch.cuda.synchronize()
    exp = O.meank_scores(means_from_sums(sums, counts), q, np.full(L, R, np.uint32), heads=Hq, kv_heads=Hkv,
                         dim=D, score_mask=np.array(mask, np.uint8), aggregation=agg, scale=1 / np.sqrt(D))
    ok, worst = within(out.cpu().numpy(), exp)
    assert ok, worst


def test_meank_add_ranges(ctx):
    import kvmem_b200 as K
    dev = torch.device("cuda", 0)
    k_d = torch.zeros(2 * 256 * 64 * 2, dtype=torch.uint8, device=dev)
    kc = K.RecallContext.make_kcache(k_d, U.F16, kv_heads=2, head_dim=64, capacity_tokens=256)
    sums_d = torch.zeros((1, 4, 128), dtype=torch.float32, device=dev)
    counts_d = torch.zeros((4,), dtype=torch.int32, device=dev)
    ctx.meank_add(kc, sums_d, counts_d, tok0=10, n=0, page_tokens=64, kv_heads=2, head_dim=64)  # no-op
    with pytest.raises(K.KvmError) as e:  # past the allocated tokens
        ctx.meank_add(kc, sums_d, counts_d, tok0=250, n=10, page_tokens=64, kv_heads=2, head_dim=64)
    assert e.value.code == K._abi.ERR_LENGTH
    with pytest.raises(K.KvmError) as e:  # past the table's pages
        ctx.meank_add(kc, sums_d, counts_d, tok0=0, n=200, page_tokens=32, kv_heads=2, head_dim=64)
    assert e.value.code == K._abi.ERR_LENGTH
    torch.cuda.synchronize()
    assert float(sums_d.abs().sum()) == 0.0 and int(counts_d.sum()) == 0
