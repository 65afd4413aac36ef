"""Seeded synthetic workloads for the benchmark configurations, generated on the device.

Config 2 (the headline): 64 layers, 24 query / 4 KV heads, head_dim 256,
131,072-token history in pages of 256 (512 pages per layer), fp16 K and V
~ N(0,1) times a per-channel scale ~ U(0.5, 2); 32 needle pages per layer whose
K rows are 0.8 * q_dir + 0.6 * N(0,1) (times the channel scale), q_dir being the
layer's mean query direction of the KV head's group normalised to unit RMS;
one decode query per head ~ N(0,1); top-32 plus first / last page kept.

Config 4 (multi-lane replay): 8 lanes x 48 layers, 40 query / 8 KV heads,
head_dim 128, 65,536 tokens per lane in pages of 128, fp16 K ~ N(0,1) times
the channel scale; 32 replayed query rows per lane; top-24 per (lane, layer,
KV head). The lanes are independent histories, so they are stacked on the
layer axis (384 rows of K and queries).

Steady-state turnover: `rotating` of the needle pages of every layer rotate.
Besides its fixed needles (K rows 0.8 * q_dir + 0.6 * N(0,1)), each layer holds
`rot_groups` groups of `rotating` pages whose K rows are 0.8 * u_j + 0.6 * N(0,1),
u_j a seeded direction of unit RMS per (layer, group, KV head). The query of decode
step s is the base query plus 0.5 * u_(s mod rot_groups) on the heads of each KV
head, so step s's group outranks the fixed needles and the other groups sit among
the noise pages: every step evicts the previous group's pages and restores the
next group's, `rotating` pages per layer (config 2: 3 of its 32 pages, about 10%).

Everything is produced by torch generators seeded per (seed, layer) so a rerun
gives the same bytes; host copies (for stage-in) are pinned and mapped.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class Workload:
    name: str
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    tokens: int
    page_tokens: int
    top_k: int
    needles: int
    keep_first_last: bool = True
    groups: int = 1          # 1: per-layer selection; kv_heads: per (layer, KV head)
    rows: int = 1            # query rows per decode step (replay rows)
    k_type: int = 1          # kvm_type of K (1 = F16, 3 = Q8_0)
    v_type: int = 1          # kvm_type of V (1 = F16, 4 = Q4_0)
    rotating: int = 0        # needle pages per layer that rotate from step to step
    rot_groups: int = 8      # rotating groups per layer (step s favours group s mod rot_groups)

    @property
    def pages(self) -> int:
        return -(-self.tokens // self.page_tokens)

    @property
    def budget(self) -> int:
        return self.top_k + (2 if self.keep_first_last else 0)

    @property
    def keep(self):
        return [0, self.pages - 1] if self.keep_first_last else []


CONFIGS = {
    "c1": Workload("c1_cpu16k", 4, 32, 8, 128, 16384, 64, 16, 8, groups=8),
    "c2": Workload("c2_fp16_128k", 64, 24, 4, 256, 131072, 256, 32, 32, rotating=3),
    "c3": Workload("c3_q8k_q4v_256k", 64, 24, 4, 256, 262144, 256, 64, 32, k_type=3, v_type=4, rotating=3),
    # 8 lanes x 48 layers folded into 384 (lane, layer) rows of independent selections.
    "c4": Workload("c4_replay_8x48x64k", 8 * 48, 40, 8, 128, 65536, 128, 24, 0, keep_first_last=False,
                   groups=8, rows=32),
    "c5": Workload("c5_q8k_sharded_1m", 64, 24, 4, 256, 1048576, 256, 128, 128, k_type=3, v_type=4,
                   rotating=12),
}


def _gen(seed: int, layer: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + layer * 7919 + 17)
    return g


ROT_QUERY = 0.5  # weight of the rotating direction in a step's query


def rot_dirs(w: Workload, seed: int, layer: int, device) -> torch.Tensor:
    """Directions of the rotating groups of one layer: [rot_groups][Hkv][D], unit RMS."""
    g = _gen(seed, 40_000 + layer, device)
    u = torch.randn((w.rot_groups, w.kv_heads, w.head_dim), generator=g, device=device)
    return u / u.pow(2).mean(dim=-1, keepdim=True).sqrt()


def make_queries(w: Workload, seed: int, device, drift_steps: int = 0, drift: float = 0.35):
    """Base queries [L][R][Hq][D] f32 and `drift_steps` per-step queries.

    With rotating needles, step s's query is the base plus ROT_QUERY * u_(s mod rot_groups)
    on the query heads of each KV head (steps 0, 1, ... of the timed loop use drifted[0],
    drifted[1], ...); without, the base plus drift * N(0,1)."""
    g = _gen(seed, 10_000, device)
    q = torch.randn((w.layers, w.rows, w.q_heads, w.head_dim), generator=g, device=device)
    if not w.rotating:
        drifted = [q + drift * torch.randn(q.shape, generator=g, device=device) for _ in range(drift_steps)]
        return q, drifted
    G = w.q_heads // w.kv_heads
    u = torch.stack([rot_dirs(w, seed, l, device) for l in range(w.layers)])  # [L][groups][Hkv][D]
    drifted = []
    for s in range(drift_steps):
        add = u[:, s % w.rot_groups].repeat_interleave(G, dim=1)  # [L][Hq][D]
        drifted.append(q + ROT_QUERY * add[:, None])
    return q, drifted


def needle_pages(w: Workload, seed: int, layer: int, device) -> torch.Tensor:
    """The fixed needle pages of one layer (sorted)."""
    return _needle_perm(w, seed, layer, device)[0]


def rotating_pages(w: Workload, seed: int, layer: int, device) -> torch.Tensor:
    """[rot_groups][rotating] pages of the rotating groups of one layer."""
    return _needle_perm(w, seed, layer, device)[1]


def _needle_perm(w: Workload, seed: int, layer: int, device):
    g = _gen(seed, 20_000 + layer, device)
    n_rot = w.rotating * w.rot_groups if w.rotating else 0
    perm = torch.randperm(w.pages - 2, generator=g, device=device)[: w.needles - w.rotating + n_rot] + 1
    fixed = torch.sort(perm[: w.needles - w.rotating]).values
    rot = perm[w.needles - w.rotating:].view(w.rot_groups, w.rotating) if n_rot else perm[:0].view(0, 0)
    return fixed, rot


def _plant(w: Workload, seed: int, layer: int, z: torch.Tensor, qd: torch.Tensor, device) -> None:
    """Needles into z [T][Hkv][D] (in place): fixed pages along q_dir, rotating groups along u_j."""
    zp = z.view(w.pages, w.page_tokens, w.kv_heads, w.head_dim)
    fixed, rot = _needle_perm(w, seed, layer, device)
    zp[fixed] = 0.8 * qd + 0.6 * zp[fixed]
    if w.rotating:
        u = rot_dirs(w, seed, layer, device)
        for j in range(w.rot_groups):
            zp[rot[j]] = 0.8 * u[j] + 0.6 * zp[rot[j]]


def fp16_layer(w: Workload, seed: int, layer: int, q: torch.Tensor, device) -> torch.Tensor:
    """K of one layer, fp16 [tokens_alloc][Hkv][D], with the layer's needle pages planted."""
    g = _gen(seed, layer, device)
    T = w.pages * w.page_tokens
    scale = torch.rand((w.kv_heads, w.head_dim), generator=g, device=device) * 1.5 + 0.5
    z = torch.randn((T, w.kv_heads, w.head_dim), generator=g, device=device)
    G = w.q_heads // w.kv_heads
    qd = q[layer].mean(dim=0).view(w.kv_heads, G, w.head_dim).mean(dim=1)  # [Hkv][D]
    qd = qd / qd.pow(2).mean(dim=-1, keepdim=True).sqrt()
    _plant(w, seed, layer, z, qd, device)
    return (z * scale).to(torch.float16)


def fp16_v_layer(w: Workload, seed: int, layer: int, device) -> torch.Tensor:
    g = _gen(seed, 30_000 + layer, device)
    T = w.pages * w.page_tokens
    scale = torch.rand((w.kv_heads, w.head_dim), generator=g, device=device) * 1.5 + 0.5
    return (torch.randn((T, w.kv_heads, w.head_dim), generator=g, device=device) * scale).to(torch.float16)


def q8_0_layer(w: Workload, seed: int, layer: int, q: torch.Tensor, device) -> torch.Tensor:
    """GGUF q8_0 K of one layer as bytes [tokens_alloc][Hkv][D/32*34]: codes
    round(N(0,1)*40) clamped to +-127 (needle rows: round(40*(0.8 q_dir + 0.6 z))), scales U(0.005, 0.03)."""
    g = _gen(seed, layer, device)
    T = w.pages * w.page_tokens
    nb = w.head_dim // 32
    z = torch.randn((T, w.kv_heads, w.head_dim), generator=g, device=device)
    G = w.q_heads // w.kv_heads
    qd = q[layer].mean(dim=0).view(w.kv_heads, G, w.head_dim).mean(dim=1)
    qd = qd / qd.pow(2).mean(dim=-1, keepdim=True).sqrt()
    _plant(w, seed, layer, z, qd, device)
    codes = torch.clamp(torch.round(z * 40), -127, 127).to(torch.int8).view(T, w.kv_heads, nb, 32)
    d = (torch.rand((T, w.kv_heads, nb), generator=g, device=device) * 0.025 + 0.005).to(torch.float16)
    out = torch.empty((T, w.kv_heads, nb, 34), dtype=torch.uint8, device=device)
    out[..., 0:2] = d.view(torch.uint8).view(T, w.kv_heads, nb, 2)
    out[..., 2:] = codes.view(torch.uint8)
    return out.view(T, w.kv_heads, nb * 34)


def q4_0_v_layer(w: Workload, seed: int, layer: int, device) -> torch.Tensor:
    g = _gen(seed, 30_000 + layer, device)
    T = w.pages * w.page_tokens
    nb = w.head_dim // 32
    out = torch.empty((T, w.kv_heads, nb, 18), dtype=torch.uint8, device=device)
    d = (torch.rand((T, w.kv_heads, nb), generator=g, device=device) * 0.025 + 0.005).to(torch.float16)
    out[..., 0:2] = d.view(torch.uint8).view(T, w.kv_heads, nb, 2)
    out[..., 2:] = torch.randint(0, 256, (T, w.kv_heads, nb, 16), generator=g, device=device, dtype=torch.uint8)
    return out.view(T, w.kv_heads, nb * 18)
