"""Tile layout restated in numpy (test oracle only).

Follows veda_comfy/core/tiling.py:
  * span_tiles        tiling.py:102-112  (box order h-block, w-block,
                      t-block; rows t,h,w row-major inside a box; real rows
                      stably compacted to the front of each tile)
  * build_tile_layout tiling.py:171-224  (video tiles of all spans, then
                      global rows chunked into 128-row tiles)
  * gather / scatter  tiling.py:227-252
"""

from __future__ import annotations

import dataclasses

import numpy as np

TILE = 128


def padded(extent: int, step: int) -> int:
    return -(-extent // step) * step


def span_tiles(start: int, grid, shape) -> np.ndarray:
    """[n_tiles, 128] int64 packed row ids of one span, -1 on padding."""
    t, h, w = grid
    st, sh, sw = shape
    if st * sh * sw != TILE:
        raise ValueError(f'tile {shape} does not hold {TILE} tokens')
    tp, hp, wp = padded(t, st), padded(h, sh), padded(w, sw)
    ids = np.full((tp, hp, wp), -1, dtype=np.int64)
    ids[:t, :h, :w] = start + np.arange(t * h * w).reshape(t, h, w)
    boxes = ids.reshape(tp // st, st, hp // sh, sh, wp // sw, sw)
    boxes = boxes.transpose(2, 4, 0, 1, 3, 5).reshape(-1, TILE)
    order = np.argsort(boxes < 0, axis=1, kind='stable')
    return np.take_along_axis(boxes, order, axis=1)


@dataclasses.dataclass
class Layout:
    """Numpy twin of `TileLayout` (tiling.py:115-168)."""

    perm: np.ndarray            # [N] int64, -1 on padding
    valid_count: np.ndarray     # [n_tiles] int32
    n_video_tiles: int
    n_ref_tiles: int
    n_global_tiles: int
    ref_tokens: int
    target_tokens: int
    seq_len: int

    @property
    def n_tiles(self) -> int:
        return self.n_video_tiles + self.n_global_tiles

    @property
    def num_slots(self) -> int:
        return self.n_tiles * TILE

    @property
    def kv_ok(self) -> np.ndarray:
        return self.valid_count > 0

    @property
    def slot_valid(self) -> np.ndarray:
        return self.perm >= 0


def build_tile_layout(spans, seq_len: int) -> Layout:
    """spans: [(start, (T, H, W), (t, h, w)), ...] in packed order, last is
    the target span."""
    if not spans:
        raise ValueError('at least the target span must be tiled')
    covered = np.zeros(seq_len, dtype=bool)
    tiles, prev = [], 0
    for start, grid, shape in spans:
        rows = grid[0] * grid[1] * grid[2]
        if start < prev or start + rows > seq_len:
            raise ValueError(f'span at {start} overlaps or exceeds {seq_len}')
        prev = start + rows
        covered[start:prev] = True
        tiles.append(span_tiles(start, grid, shape))
    n_ref = sum(t.shape[0] for t in tiles[:-1])
    video = np.concatenate(tiles)
    global_rows = np.nonzero(~covered)[0]
    n_global = -(-global_rows.size // TILE)
    gtiles = np.full(n_global * TILE, -1, dtype=np.int64)
    gtiles[:global_rows.size] = global_rows
    perm = np.concatenate([video.reshape(-1), gtiles])
    valid = (perm.reshape(-1, TILE) >= 0).sum(1).astype(np.int32)
    return Layout(perm=perm, valid_count=valid, n_video_tiles=video.shape[0],
                  n_ref_tiles=n_ref, n_global_tiles=n_global,
                  ref_tokens=sum(g[0] * g[1] * g[2] for _, g, _ in spans[:-1]),
                  target_tokens=int(np.prod(spans[-1][1])), seq_len=seq_len)


def identity_layout(seq_len: int, real: int | None = None) -> Layout:
    """One target span covering [0, real) tile-ordered as-is (the synthetic
    configs: 1 x 1 x L grid, tile 1 x 1 x 128), padded to whole tiles."""
    real = seq_len if real is None else real
    n_tiles = -(-real // TILE)
    perm = np.arange(n_tiles * TILE, dtype=np.int64)
    perm[real:] = -1
    valid = (perm.reshape(-1, TILE) >= 0).sum(1).astype(np.int32)
    return Layout(perm=perm, valid_count=valid, n_video_tiles=n_tiles,
                  n_ref_tiles=0, n_global_tiles=0, ref_tokens=0,
                  target_tokens=real, seq_len=real)


def gather_tiles(x: np.ndarray, layout: Layout) -> np.ndarray:
    """[S, H, D] -> [N, H, D] tile order, padding rows zero."""
    out = x[np.clip(layout.perm, 0, None)].copy()
    out[layout.perm < 0] = 0
    return out


def scatter_tiles(tiled: np.ndarray, layout: Layout) -> np.ndarray:
    """[N, H, D] -> [S, H, D]; padding slots are dropped."""
    out = np.zeros((layout.seq_len,) + tiled.shape[1:], dtype=tiled.dtype)
    real = layout.perm >= 0
    out[layout.perm[real]] = tiled[real]
    return out
