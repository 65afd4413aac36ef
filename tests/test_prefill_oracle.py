"""CPU: the FP64 restatement of prefill attention with page-LSE capture (oracle.prefill_attention,
oracle.page_mass_from_lse) against a direct computation on a small case: causal softmax attention
row by row, the page LSE as log of the summed page probabilities times the row's partition sum,
-inf past each sampled row's causal frontier, and page masses that sum to one."""
import numpy as np

from oracle import oracle as O


def test_prefill_oracle_small_case():
    rng = np.random.default_rng(3)
    base, width, hq, hkv, dim, pt = 37, 29, 4, 2, 16, 8
    T = base + width
    q = rng.standard_normal((width, hq, dim))
    k = rng.standard_normal((T, hkv, dim))
    v = rng.standard_normal((T, hkv, dim))
    rows = [0, 5, 28]
    samples = [0, 13, 28]
    pages = -(-T // pt) + 2  # two spare columns stay -inf
    out, lse = O.prefill_attention(q, k, v, base=base, rows=rows, sample_rows=samples, page_tokens=pt, pages=pages)
    sc = 1.0 / np.sqrt(dim)
    for i, r in enumerate(rows):
        for h in range(hq):
            kv = h // (hq // hkv)
            s = sc * k[: base + r + 1, kv] @ q[r, h]
            p = np.exp(s - s.max())
            np.testing.assert_allclose(out[i, h], (p / p.sum()) @ v[: base + r + 1, kv], rtol=1e-12, atol=1e-12)
    for i, r in enumerate(samples):
        n = base + r + 1
        for h in range(hq):
            kv = h // (hq // hkv)
            s = sc * k[:n, kv] @ q[r, h]
            z = np.log(np.exp(s).sum())
            for pg in range(pages):
                blk = s[pg * pt:min(n, (pg + 1) * pt)]
                if pg * pt >= n:
                    assert lse[i, h, pg] == -np.inf
                else:
                    np.testing.assert_allclose(lse[i, h, pg], np.log(np.exp(blk).sum()), rtol=1e-12, atol=1e-12)
            # exp(page LSE) over all pages is the row's partition sum
            np.testing.assert_allclose(np.log(np.exp(lse[i, h][np.isfinite(lse[i, h])]).sum()), z, rtol=1e-12)
    mass = O.page_mass_from_lse(lse)
    assert mass.shape == (len(samples), pages)
    np.testing.assert_allclose(mass.sum(axis=1), 1.0, rtol=1e-12)
    assert (mass[:, -2:] == 0).all()
