"""Tile layouts: every 128 permuted rows form one 3-D tile of a span.

Same contract as the reference's `core/tiling.py` (the one its released
predictors were trained on): a (t, h, w) tile shape with t*h*w = 128 cuts a
span's (T, H, W) grid into boxes, box order (h-block, w-block, t-block)
outer to inner, rows t, h, w row-major inside a box, real rows stably
compacted to the front, so a tile's real rows are a prefix of length
`valid_count[tile]` (tiling.py:102-112). Rows outside every span are
global: chunked into 128-row tiles in sequence order after all span tiles
(tiling.py:171-224).

Layouts are built once per geometry on the host; `gather_tiles` and
`scatter_tiles_` run on the GPU (csrc/tiling.cu). `TileLayout` carries the
attribute names of the reference's layout object, so a reference layout can
be passed to this package's ops unchanged.
"""

from __future__ import annotations

import dataclasses
from collections.abc import Sequence

import numpy as np
import torch

from . import ops

TILE_SIZE = 128


@dataclasses.dataclass(frozen=True, order=True)
class TileShape:
    """The extents (t, h, w) of one tile in frames, rows and columns of the
    latent grid; their product is the tile size, 128."""

    t: int
    h: int
    w: int

    def __post_init__(self):
        if self.t * self.h * self.w != TILE_SIZE:
            raise ValueError(f'{self.t} x {self.h} x {self.w} is '
                             f'{self.t * self.h * self.w} tokens; a tile has '
                             f'{TILE_SIZE}')

    def padded_grid(self, grid: Sequence[int]) -> tuple[int, int, int]:
        """`grid` rounded up, per axis, to a whole number of tiles."""
        return tuple(-(-g // s) * s
                     for g, s in zip(grid, (self.t, self.h, self.w)))

    def num_tiles(self, grid: Sequence[int]) -> int:
        """Tiles that cover `grid`, padding included."""
        tp, hp, wp = self.padded_grid(grid)
        return tp * hp * wp // TILE_SIZE


@dataclasses.dataclass(frozen=True)
class TiledSpan:
    """A video span of the packed sequence: T * H * W consecutive rows from
    `start`, frame-major then row-major, cut into tiles of `shape`."""

    start: int
    grid: tuple[int, int, int]
    shape: TileShape

    @property
    def num_rows(self) -> int:
        t, h, w = self.grid
        return t * h * w


def span_tiles(span: TiledSpan) -> np.ndarray:
    """The packed rows of each tile of a span, [n_tiles, 128] int64. Tiles
    are numbered h-block, w-block, t-block from outer to inner; inside a
    tile the real rows come first in (t, h, w) order and the padding (-1)
    last."""
    t, h, w = span.grid
    s = span.shape
    tp, hp, wp = s.padded_grid(span.grid)
    ids = np.full((tp, hp, wp), -1, dtype=np.int64)
    ids[:t, :h, :w] = span.start + np.arange(t * h * w).reshape(t, h, w)
    boxes = ids.reshape(tp // s.t, s.t, hp // s.h, s.h, wp // s.w, s.w)
    boxes = boxes.transpose(2, 4, 0, 1, 3, 5).reshape(-1, TILE_SIZE)
    real_first = np.argsort(boxes < 0, axis=1, kind='stable')
    return np.take_along_axis(boxes, real_first, axis=1)


@dataclasses.dataclass
class TileLayout:
    """One permutation of the packed sequence and its derived constants
    (attribute names of the reference's TileLayout, tiling.py:115-168)."""

    perm: torch.Tensor            # [N] int64, -1 on padding
    valid_count: torch.Tensor     # [n_tiles] int32
    n_video_tiles: int
    n_ref_tiles: int
    n_global_tiles: int
    ref_tokens: int
    target_tokens: int
    seq_len: int
    kv_ok: torch.Tensor           # [n_tiles] bool
    slot_valid: torch.Tensor      # [N] int32
    identity: bool = False        # perm is 0..N-1 over real rows
    n_global_ok: int = 0          # non-empty global tiles (host copy)

    @property
    def n_tiles(self) -> int:
        return self.n_video_tiles + self.n_global_tiles

    @property
    def num_slots(self) -> int:
        return self.n_tiles * TILE_SIZE


def _layout(perm: np.ndarray, n_video: int, n_ref: int, n_global: int,
            ref_tokens: int, target_tokens: int, seq_len: int,
            device) -> TileLayout:
    valid = (perm.reshape(-1, TILE_SIZE) >= 0).sum(1).astype(np.int32)
    real = perm >= 0
    identity = bool(np.array_equal(perm[real], np.arange(real.sum())))
    return TileLayout(
        perm=torch.from_numpy(perm).to(device),
        valid_count=torch.from_numpy(valid).to(device),
        n_video_tiles=n_video, n_ref_tiles=n_ref, n_global_tiles=n_global,
        ref_tokens=ref_tokens, target_tokens=target_tokens, seq_len=seq_len,
        kv_ok=torch.from_numpy(valid > 0).to(device),
        slot_valid=torch.from_numpy(real.astype(np.int32)).to(device),
        identity=identity and bool(real[:real.sum()].all()),
        n_global_ok=int((valid[n_video:] > 0).sum()))


def build_tile_layout(spans: Sequence[TiledSpan], seq_len: int,
                      device: torch.device | str = 'cpu') -> TileLayout:
    """The permutation of `spans` (packed order, the last is the target);
    rows outside every span are global.

    Raises:
        ValueError: If spans overlap, are out of order or exceed seq_len.
    """
    if not spans:
        raise ValueError('at least the target span must be tiled')
    covered = np.zeros(seq_len, dtype=bool)
    tiles, prev = [], 0
    for span in spans:
        stop = span.start + span.num_rows
        if span.start < prev or stop > seq_len:
            raise ValueError(f'span {span} overlaps or exceeds {seq_len}')
        prev = stop
        covered[span.start:stop] = True
        tiles.append(span_tiles(span))
    video = np.concatenate(tiles)
    global_rows = np.flatnonzero(~covered)
    n_global = -(-global_rows.size // TILE_SIZE)
    tail = np.full(n_global * TILE_SIZE, -1, dtype=np.int64)
    tail[:global_rows.size] = global_rows
    perm = np.concatenate([video.reshape(-1), tail])
    return _layout(perm, video.shape[0], sum(t.shape[0] for t in tiles[:-1]),
                   n_global, sum(s.num_rows for s in spans[:-1]),
                   spans[-1].num_rows, seq_len, device)


def identity_layout(real_tokens: int,
                    device: torch.device | str = 'cpu') -> TileLayout:
    """Rows already in tile order: one 1 x 1 x L target span tiled
    1 x 1 x 128, padded to whole tiles (the synthetic benchmark layout)."""
    n_tiles = -(-real_tokens // TILE_SIZE)
    perm = np.arange(n_tiles * TILE_SIZE, dtype=np.int64)
    perm[real_tokens:] = -1
    return _layout(perm, n_tiles, 0, 0, 0, real_tokens, real_tokens, device)


def from_reference(layout, device: torch.device | str | None = None
                   ) -> TileLayout:
    """This package's TileLayout from the reference's own (core/tiling.py:
    115-168): the same permutation and tile counts; the reference's derived
    index tensors (gather_index, scatter_index, ...) are not needed here.
    Reads `perm` once on the host, so convert once per geometry."""
    perm = layout.perm.detach().to('cpu', torch.int64).numpy()
    device = layout.perm.device if device is None else device
    return _layout(perm, int(layout.n_video_tiles), int(layout.n_ref_tiles),
                   int(layout.n_global_tiles), int(layout.ref_tokens),
                   int(layout.target_tokens), int(layout.seq_len), device)


def gather_tiles(x: torch.Tensor, layout, heads: torch.Tensor) -> torch.Tensor:
    """[S, H, D] packed -> [N, H', D] contiguous tile order, padding zero."""
    return ops.gather_tiles(x, layout.perm, heads)


def scatter_tiles_(out: torch.Tensor, tiled: torch.Tensor, layout,
                   heads: torch.Tensor) -> None:
    """Writes tile-ordered rows back into out[S(+1), H, D] in place; padding
    slots are dropped."""
    ops.scatter_tiles_(out, tiled, layout.perm, heads)
