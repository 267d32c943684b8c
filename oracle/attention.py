"""Exact fp32 masked block-sparse attention in numpy (test oracle only).

Follows veda_comfy/core/reference.py:14-36 (`block_sparse_attention`): the
block mask is expanded to token level, key slots that are padding are
masked, softmax in fp32 (rows with nothing allowed give 0), padding query
rows are zeroed. Computed one head at a time to bound memory, as the
reference's CPU baseline is run at long sequence lengths.
"""

from __future__ import annotations

import numpy as np

TILE = 128


def mask_from_lists(index: np.ndarray, count: np.ndarray,
                    n_tiles: int) -> np.ndarray:
    """[H, n, W] index lists + [H, n] counts -> [H, n, n] bool mask."""
    heads, n = count.shape
    mask = np.zeros((heads, n, n_tiles), dtype=bool)
    live = np.arange(index.shape[-1])[None, None, :] < count[..., None]
    h, r, c = np.nonzero(live)
    mask[h, r, index[h, r, c]] = True
    return mask


def block_sparse_head(q, k, v, mask_h, slot_valid, rows=None):
    """One head: q/k/v [N, D] fp32, mask_h [n, n] bool -> [N or len(rows), D]
    fp32. `rows` limits the query rows (a bounded sample)."""
    scale = np.float32(q.shape[-1] ** -0.5)
    rows = np.arange(q.shape[0]) if rows is None else np.asarray(rows)
    allowed = np.repeat(mask_h[rows // TILE], TILE, axis=1)
    allowed &= slot_valid[None, :]
    scores = (q[rows] @ k.T) * scale
    scores = np.where(allowed, scores, -np.inf).astype(np.float32)
    m = scores.max(axis=1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
    e = np.exp(scores - m)
    denom = e.sum(axis=1, keepdims=True)
    probs = np.where(denom > 0, e / np.where(denom > 0, denom, 1), 0.0)
    out = probs.astype(np.float32) @ v
    return out * slot_valid[rows, None].astype(np.float32)


def block_sparse_attention(q, k, v, mask, slot_valid, heads=None):
    """q/k/v [N, H, D] (any float dtype), mask [H, n, n] -> fp32 [N, H, D]."""
    n, n_heads, dim = q.shape
    out = np.zeros((n, n_heads, dim), dtype=np.float32)
    for h in (range(n_heads) if heads is None else heads):
        out[:, h] = block_sparse_head(
            q[:, h].astype(np.float32), k[:, h].astype(np.float32),
            v[:, h].astype(np.float32), mask[h], slot_valid)
    return out
