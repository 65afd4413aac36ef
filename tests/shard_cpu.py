"""numpy stand-ins for the five per-rank compute steps of sharded selection
(the kernels' semantics), used to run the exchange logic on gloo ranks on CPU."""
import numpy as np
import torch


def lse_pages(q, k, tokens, page_tokens, scale, page0, local_pages):
    """q [L][R][Hq][D] f64, k [L][T][Hkv][D] f64 (full history) -> local LSE [L][R][Hq][local_pages]."""
    L, R, Hq, D = q.shape
    Hkv = k.shape[2]
    G = Hq // Hkv
    out = np.full((L, R, Hq, local_pages), -np.inf)
    for l in range(L):
        for r in range(R):
            for h in range(Hq):
                for pp in range(local_pages):
                    t0 = (page0 + pp) * page_tokens
                    t1 = min(t0 + page_tokens, tokens)
                    if t1 <= t0:
                        continue
                    x = k[l, t0:t1, h // G] @ q[l, r, h] * scale
                    m = x.max()
                    out[l, r, h, pp] = m + np.log(np.exp(x - m).sum())
    return out


class CpuShardCompute:
    def __init__(self, q, k, tokens, page_tokens, scale):
        self.q, self.k, self.tokens, self.B, self.scale = q, k, tokens, page_tokens, scale
        self.lse = None

    def partial(self, desc, q, k, geo):
        self.lse = lse_pages(self.q, self.k, self.tokens, self.B, self.scale, geo.page0, geo.local_pages)
        m = self.lse.max(axis=-1)
        s = np.where(np.isfinite(m), np.exp(self.lse - m[..., None]).sum(axis=-1), 0.0)
        return torch.tensor(np.stack([m, s], -1).reshape(-1, 2), dtype=torch.float64)

    def merge_stats(self, gathered, world, geo):
        g = gathered.numpy()
        M = g[..., 0].max(axis=0)
        S = (g[..., 1] * np.exp(g[..., 0] - M)).sum(axis=0)
        return torch.tensor(np.stack([M, 1 / S], -1))

    def finish(self, desc, geo, global_stats):
        st = global_stats.numpy().reshape(geo.layers, geo.rows, geo.q_heads, 2)
        prob = np.exp(self.lse - st[..., 0:1]) * st[..., 1:2]  # [L][R][Hq][P]
        return torch.tensor(prob.mean(axis=2).mean(axis=1))  # groups == 1: mean over heads, then rows

    def candidates(self, mass, geo, keep, k):
        m = mass.numpy()
        cs = np.full((geo.sel_rows, k), -np.inf)
        ci = np.full((geo.sel_rows, k), -1, np.int64)
        for row in range(geo.sel_rows):
            cand = [(m[row, p], geo.page0 + p) for p in range(geo.local_pages) if geo.page0 + p not in keep]
            cand.sort(key=lambda x: (-x[0], -x[1]))
            cand = sorted(cand[:k], key=lambda x: x[1])
            for i, (s, g) in enumerate(cand):
                cs[row, i], ci[row, i] = s, g
        return torch.tensor(cs), torch.tensor(ci)

    def merge(self, gs, gi, world, geo, keep, k, budget):
        gs, gi = gs.numpy(), gi.numpy()
        ids = np.zeros((geo.sel_rows, budget), np.int64)
        n = np.zeros(geo.sel_rows, np.int64)
        for row in range(geo.sel_rows):
            cand = [(gs[r, row, j], gi[r, row, j]) for r in range(world) for j in range(k) if gi[r, row, j] >= 0]
            cand.sort(key=lambda x: (-x[0], -x[1]))
            chosen = sorted(set(keep) | {g for _, g in cand[: budget - len(keep)]})
            ids[row, : len(chosen)] = chosen
            n[row] = len(chosen)
        return torch.tensor(ids), torch.tensor(n)

    # The one-collective strategy (LseGatherSelector): local LSE, whole-row masses, top-k.
    def page_lse(self, desc, q, k, geo):
        return torch.tensor(lse_pages(self.q, self.k, self.tokens, self.B, self.scale, geo.page0, geo.local_pages))

    def mass_from_lse(self, desc, geo, lse):
        x = lse.numpy()  # [L][R][Hq][P]
        m = x.max(axis=-1, keepdims=True)
        prob = np.exp(x - m) / np.exp(x - m).sum(axis=-1, keepdims=True)
        return torch.tensor(prob.mean(axis=2).mean(axis=1))  # groups == 1

    def select_topk(self, mass, keep, budget):
        from oracle import oracle as O
        m = mass.numpy()
        ids = np.zeros((m.shape[0], budget), np.int64)
        n = np.zeros(m.shape[0], np.int64)
        for row in range(m.shape[0]):
            rc, got = O.pick_scored(m.shape[1], list(range(m.shape[1])), m[row], keep, budget)
            assert rc == 0
            ids[row, : len(got)] = got
            n[row] = len(got)
        return torch.tensor(ids), torch.tensor(n)
