"""Veda predictor tile scoring on the GPU.

Same arithmetic as the reference's core/predictor.py: TripPool features
[mean | max | min] over the real rows of every video tile (:20-60), and
block logits q_hat k_hat^T / sqrt(D) with x_hat = F @ P[h] + F[:, :D]
(:63-80), all fp32. In the engine the pooling is fused into the Q / K
quantisation pass (ops.quant_pool); `pool_video_tiles` is the standalone
form of the same kernel.
"""

from __future__ import annotations

import torch

from . import ops


def pool_video_tiles(x: torch.Tensor, layout) -> torch.Tensor:
    """[N, H', D] tile-ordered -> [H', n_video_tiles, 3D] fp32 features;
    exactly 0 for empty tiles."""
    feats = ops.quant_pool(x, x, layout.valid_count, layout.n_video_tiles,
                           1.0, pool=True)
    return feats['feats_q']


def tile_logits(feats_q: torch.Tensor, feats_k: torch.Tensor,
                proj_q: torch.Tensor, proj_k: torch.Tensor,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """[H', n_q, 3D] x [H', n_k, 3D] features, [H', 3D, D] projections ->
    [H', n_q, n_k] fp32 logits."""
    return ops.tile_logits(feats_q, feats_k, proj_q, proj_k, workspace)
