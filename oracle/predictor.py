"""Predictor tile scoring restated in numpy (test oracle only).

Follows veda_comfy/core/predictor.py:
  * pool_video_tiles  predictor.py:20-60  masked mean (sum / max(count, 1)),
                      max and min over the real (prefix) rows of every video
                      tile -> [H, n_video, 3D]; 0 for empty tiles.
  * tile_logits       predictor.py:63-80  x_hat = F @ P[h] + F[:, :D];
                      logits = q_hat k_hat^T / sqrt(D).

Accumulates in float64 so it is at least as accurate as the reference's
fp32 sums; comparisons against it use a tolerance.
"""

from __future__ import annotations

import math

import numpy as np

from . import tiling


def pool_video_tiles(x: np.ndarray, layout: tiling.Layout) -> np.ndarray:
    """x: [N, H, D] tile-ordered (any float dtype) -> [H, n_video, 3D] f32."""
    n = layout.n_video_tiles
    heads, dim = x.shape[1], x.shape[2]
    tiles = x[:n * tiling.TILE].astype(np.float64).reshape(
        n, tiling.TILE, heads, dim)
    valid = np.arange(tiling.TILE)[None, :] < layout.valid_count[:n, None]
    live = valid[:, :, None, None]
    count = np.maximum(layout.valid_count[:n], 1).astype(np.float64)
    mean = np.where(live, tiles, 0.0).sum(1) / count[:, None, None]
    tmax = np.where(live, tiles, -np.inf).max(1)
    tmin = np.where(live, tiles, np.inf).min(1)
    feats = np.concatenate([mean, tmax, tmin], axis=-1)
    feats = np.where(layout.kv_ok[:n, None, None], feats, 0.0)
    return feats.transpose(1, 0, 2).astype(np.float32)


def tile_logits(feats_q, feats_k, proj_q, proj_k) -> np.ndarray:
    """feats [H, n, 3D] f32, proj [H, 3D, D] -> [H, n_q, n_k] f32."""
    dim = proj_q.shape[-1]
    fq, fk = feats_q.astype(np.float64), feats_k.astype(np.float64)
    q_hat = fq @ proj_q.astype(np.float64) + fq[..., :dim]
    k_hat = fk @ proj_k.astype(np.float64) + fk[..., :dim]
    return (q_hat @ k_hat.transpose(0, 2, 1) / math.sqrt(dim)).astype(
        np.float32)
