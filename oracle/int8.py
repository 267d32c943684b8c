"""The reference INT8 arithmetic restated in numpy (test oracle only).

Follows veda_comfy/kernels/sage/sparse_int8.py:
  * quantize   sparse_int8.py:57-73, 118-133: x = x * pre_scale (fp32);
               scale = max|x| / 127 per (block of rows, head), 1.0 when the
               block is all zero; q = x / scale; q += 0.5 * sign (>= 0 counts
               as positive); int8 = trunc(q). All fp32 with IEEE division.
  * attend     sparse_int8.py:312-362: Q per 128 rows with
               pre_scale = D^-0.5 * log2(e); K per 64 rows; logits in base 2
               are int32(Qi8 . Ki8) * q_scale * k_scale; key columns at or
               past the tile's valid count are masked.
  * key_blocks sparse_int8.py:295-309 (128-row tiles -> 64-row key blocks)

`int8_block_sparse` computes the softmax of those logits exactly (float64),
optionally rounding P to a 16-bit type the way a kernel feeding P to a
16-bit tensor-core product does; it is the arithmetic the kernel has to
reproduce, independent of the kernel's own summation order.
"""

from __future__ import annotations

import numpy as np

TILE = 128
KEY_BLOCK = 64
LOG2E = 1.4426950408889634


def q_pre_scale(dim: int, softmax_scale: float | None = None) -> np.float32:
    """The factor folded into Q before quantising (sparse_int8.py:330,336),
    as the fp32 the Triton launch passes."""
    scale = dim ** -0.5 if softmax_scale is None else softmax_scale
    return np.float32(scale * LOG2E)


def quantize(x: np.ndarray, block: int, pre_scale=1.0):
    """[N, H, D] -> (int8 [N, H, D], fp32 scales [H, N // block])."""
    n, heads, dim = x.shape
    x32 = x.astype(np.float32) * np.float32(pre_scale)
    xb = x32.reshape(n // block, block, heads, dim)
    amax = np.abs(xb).max(axis=(1, 3))                     # [nb, H]
    scale = (amax / np.float32(127.0)).astype(np.float32)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = (xb / scale[:, None, :, None]).astype(np.float32)
    q = (q + np.where(q >= 0, np.float32(0.5), np.float32(-0.5))).astype(
        np.float32)
    qi = np.trunc(q).astype(np.int8)
    return qi.reshape(n, heads, dim), np.ascontiguousarray(scale.T)


def key_blocks(index: np.ndarray, count: np.ndarray,
               valid_count: np.ndarray, block: int = KEY_BLOCK):
    sub = TILE // block
    blocks = (index.astype(np.int32)[..., None] * sub
              + np.arange(sub, dtype=np.int32)).reshape(*index.shape[:-1], -1)
    valid = np.clip(valid_count[:, None] - np.arange(sub) * block, 0, block)
    return blocks, (count * sub).astype(np.int32), valid.reshape(-1).astype(
        np.int32)


def _round16(p: np.ndarray, kind: str | None) -> np.ndarray:
    if kind is None:
        return p
    if kind == 'f16':
        return p.astype(np.float16).astype(np.float64)
    if kind == 'bf16':
        f = p.astype(np.float32)
        bits = f.view(np.uint32).astype(np.uint64)
        bits = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
        return bits.astype(np.uint32).view(np.float32).astype(np.float64)
    raise ValueError(kind)


def int8_block_sparse(q, k, v, index, count, valid_count,
                      softmax_scale=None, p_round: str | None = None,
                      heads=None, q_tiles=None):
    """INT8 block-sparse attention on tile-ordered [N, H, D] inputs.

    index [H, n_tiles, W] ascending kept tile ids, count [H, n_tiles].
    Returns float64 [N, H, D]; query tiles with count 0 give zeros.
    `heads` / `q_tiles` restrict the work to a sample (other rows stay 0).
    """
    n, n_heads, dim = q.shape
    qi, qs = quantize(q, TILE, q_pre_scale(dim, softmax_scale))
    ki, ks = quantize(k, KEY_BLOCK)
    vf = v.astype(np.float64)
    out = np.zeros((n, n_heads, dim), dtype=np.float64)
    col_in_tile = np.arange(TILE)
    for h in (range(n_heads) if heads is None else heads):
        for qt in (range(n // TILE) if q_tiles is None else q_tiles):
            c = int(count[h, qt])
            if c == 0:
                continue
            tiles = index[h, qt, :c].astype(np.int64)
            keys = (tiles[:, None] * TILE + col_in_tile).reshape(-1)
            rows = slice(qt * TILE, (qt + 1) * TILE)
            s_int = qi[rows, h].astype(np.int32) @ ki[keys, h].astype(
                np.int32).T
            s = (s_int.astype(np.float32) * qs[h, qt]
                 * ks[h, keys // KEY_BLOCK][None, :]).astype(np.float64)
            live = (valid_count[tiles][:, None] > col_in_tile).reshape(-1)
            s[:, ~live] = -np.inf
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            p = np.exp2(s - m)
            l_sum = p.sum(axis=1, keepdims=True)
            p = _round16(p, p_round)
            acc = p @ vf[keys, h]
            out[rows, h] = acc / np.where(l_sum > 0, l_sum, 1.0)
    return out

