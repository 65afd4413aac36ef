"""Seeded synthetic inputs for the tests (host numpy; uploaded as raw bytes)."""
from __future__ import annotations

import numpy as np

F32, F16, BF16, Q8_0, Q4_0, Q5_0 = 0, 1, 2, 3, 4, 5
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q5_0: 22}


def row_bytes(ktype: int, dim: int) -> int:
    if ktype == F32:
        return 4 * dim
    if ktype in (F16, BF16):
        return 2 * dim
    return dim // 32 * BLOCK_BYTES[ktype]


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def encode(vals: np.ndarray, ktype: int) -> np.ndarray:
    """f32 values [..., D] -> bytes [..., row_bytes] of ktype (float types only)."""
    if ktype == F32:
        return np.ascontiguousarray(vals, np.float32).view(np.uint8)
    if ktype == F16:
        return np.ascontiguousarray(vals.astype(np.float16)).view(np.uint8)
    if ktype == BF16:
        return to_bf16_bits(vals).view(np.uint8)
    raise ValueError(ktype)


def make_quant_rows(rng, ktype: int, nrows: int, dim: int) -> np.ndarray:
    """Random GGUF blocks: q8_0 codes round(N(0,1)*40) clamped to +-127, scales U(0.005,0.03)."""
    nb = dim // 32
    out = np.zeros((nrows, nb, BLOCK_BYTES[ktype]), np.uint8)
    d = rng.uniform(0.005, 0.03, (nrows, nb)).astype(np.float16)
    out[:, :, 0:2] = d.view(np.uint8).reshape(nrows, nb, 2)
    if ktype == Q8_0:
        qs = np.clip(np.round(rng.standard_normal((nrows, nb, 32)) * 40), -127, 127).astype(np.int8)
        out[:, :, 2:] = qs.view(np.uint8)
    elif ktype == Q4_0:
        out[:, :, 2:] = rng.integers(0, 256, (nrows, nb, 16), dtype=np.uint8)
    else:
        out[:, :, 2:] = rng.integers(0, 256, (nrows, nb, 20), dtype=np.uint8)
    return out.reshape(nrows, nb * BLOCK_BYTES[ktype])


def make_k(rng, ktype: int, layers: int, tokens: int, kv_heads: int, dim: int, needle_pages=(), page=64,
           q_dir=None) -> np.ndarray:
    """K history bytes [layers, tokens, kv_heads, row_bytes]."""
    if ktype in (Q8_0, Q4_0, Q5_0):
        raw = make_quant_rows(rng, ktype, layers * tokens * kv_heads, dim)
        return raw.reshape(layers, tokens, kv_heads, -1)
    vals = rng.standard_normal((layers, tokens, kv_heads, dim)).astype(np.float32)
    if q_dir is not None:
        for p in needle_pages:
            sl = slice(p * page, (p + 1) * page)
            vals[:, sl] = 0.8 * q_dir[:, None, :, :] * np.sqrt(dim) + 0.6 * vals[:, sl]
    return encode(vals, ktype).reshape(layers, tokens, kv_heads, -1)


def make_q(rng, qtype: int, layers: int, rows: int, heads: int, dim: int) -> np.ndarray:
    """Query bytes [layers, rows, heads, dim*esize]."""
    vals = rng.standard_normal((layers, rows, heads, dim)).astype(np.float32)
    return encode(vals, qtype).reshape(layers, rows, heads, -1)


def close(actual, expected, rel=1e-3, abs_=1e-6):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    err = np.abs(actual - expected)
    bound = abs_ + rel * np.abs(expected)
    bad = ~(err <= bound)
    return not bad.any(), float(err.max(initial=0.0)), int(bad.sum())


def decode_rows_f32(kb: np.ndarray, ktype: int, dim: int) -> np.ndarray:
    """Key bytes [..., row_bytes] -> float32 [..., dim], independently of the oracle: f32/f16/bf16
    values as they are, GGUF q8_0 / q4_0 / q5_0 codes times the block's fp16 scale as one float32
    product (the reference's key(), src/adapter/llama-kvmem-attention-cuda.cu:39-58)."""
    lead = kb.shape[:-1]
    rb = row_bytes(ktype, dim)
    flat = np.ascontiguousarray(kb).reshape(-1, rb)
    if ktype == F32:
        out = flat.view(np.float32)
    elif ktype == F16:
        out = flat.view(np.float16).astype(np.float32)
    elif ktype == BF16:
        out = (flat.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    else:
        nb = dim // 32
        blocks = flat.reshape(-1, nb, BLOCK_BYTES[ktype])
        scale = blocks[..., 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
        if ktype == Q8_0:
            codes = blocks[..., 2:34].view(np.int8).astype(np.float32)
        else:
            qs = blocks[..., -16:]
            low = np.concatenate([qs & 15, qs >> 4], axis=-1).astype(np.int32)
            if ktype == Q4_0:
                codes = (low - 8).astype(np.float32)
            else:
                qh = blocks[..., 2:6].copy().view(np.uint32)[..., 0]
                high = ((qh[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int32)
                codes = ((low | (high << 4)) - 16).astype(np.float32)
        out = (codes * scale[..., None]).astype(np.float32).reshape(-1, dim)
    return out.reshape(*lead, dim)


def restore_k_numpy(ktype: int, src: np.ndarray, tokens: int, n_head: int, dim: int, n_rot: int = 0, pos0: int = 0,
                    theta=None, nrot: int = 0) -> np.ndarray:
    """Independent numpy restatement of the raw-K restore transform (float32
    arithmetic in the reference's order; sin / cos from numpy in float32)."""
    n_embd = n_head * dim
    row = decode_rows_f32(np.ascontiguousarray(src).reshape(tokens, -1), ktype, n_embd).astype(np.float32)
    if n_rot:
        half = n_rot // 2
        th = np.asarray(theta[:half], np.float32)
        pos = (np.arange(tokens, dtype=np.int64) + pos0).astype(np.float32)
        ang = (pos[:, None] * th[None, :]).astype(np.float32)
        sn, cs = np.sin(ang).astype(np.float32), np.cos(ang).astype(np.float32)
        r = row.reshape(tokens, n_head, dim)
        x0, x1 = r[:, :, :half].copy(), r[:, :, half:n_rot].copy()
        r[:, :, :half] = (x0 * cs[:, None, :]).astype(np.float32) - (x1 * sn[:, None, :]).astype(np.float32)
        r[:, :, half:n_rot] = (x0 * sn[:, None, :]).astype(np.float32) + (x1 * cs[:, None, :]).astype(np.float32)
        row = r.reshape(tokens, n_embd)
    if nrot:
        row = (row * np.float32(1.0 / np.sqrt(np.float32(nrot)))).astype(np.float32)
        c = row.reshape(tokens, n_embd // nrot, nrot)
        h = 1
        while h < nrot:
            c = c.reshape(tokens, n_embd // nrot, nrot // (2 * h), 2, h)
            a, b = c[:, :, :, 0, :].copy(), c[:, :, :, 1, :].copy()
            c[:, :, :, 0, :], c[:, :, :, 1, :] = a + b, a - b
            c = c.reshape(tokens, n_embd // nrot, nrot)
            h *= 2
        row = c.reshape(tokens, n_embd)
    blocks = row.reshape(tokens, n_embd // 32, 32)
    out = np.zeros((tokens, n_embd // 32, BLOCK_BYTES[ktype]), np.uint8)
    if ktype == Q8_0:
        d = (np.abs(blocks).max(axis=-1) / np.float32(127)).astype(np.float32)
        inv = np.where(d != 0, (np.float32(1) / np.where(d != 0, d, 1)).astype(np.float32), 0).astype(np.float32)
        x = (blocks * inv[..., None]).astype(np.float32)
        ax = np.abs(x)
        q = np.floor(ax)
        q = (q + ((ax - q) >= 0.5)) * np.sign(x)
        out[..., 0:2] = d.astype(np.float16)[..., None].view(np.uint8).reshape(tokens, -1, 2)
        out[..., 2:] = q.astype(np.int8).view(np.uint8)
    else:
        idx = np.abs(blocks).argmax(axis=-1)  # first of the largest magnitudes
        vmax = np.take_along_axis(blocks, idx[..., None], -1)[..., 0]
        d = (vmax / np.float32(-8)).astype(np.float32)
        inv = np.where(d != 0, (np.float32(1) / np.where(d != 0, d, 1)).astype(np.float32), 0).astype(np.float32)
        xi = np.minimum(np.trunc((blocks * inv[..., None]).astype(np.float32) + np.float32(8.5)), 15).astype(np.int32)
        out[..., 0:2] = d.astype(np.float16)[..., None].view(np.uint8).reshape(tokens, -1, 2)
        out[..., 2:] = ((xi[..., :16] & 15) | ((xi[..., 16:] & 15) << 4)).astype(np.uint8)
    return out.reshape(-1)
