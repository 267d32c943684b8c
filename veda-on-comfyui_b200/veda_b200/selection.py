"""Veda selection rules with the top-k and the list building on the GPU.

Host rules, same as the reference's core/selection.py: `Budget` (:39-78),
`split_budget` (:81-89), `bresenham_extra` (:92-106), `ColumnBlock` and
`column_blocks` (:109-128). The device part replaces `select` (:132-180),
`block_mask` (:184-203) and `tile_index_list` (:206-227) with one kernel
(csrc/select.cu) that writes each query tile's kept key tiles as an
ascending, -1 padded list of a width fixed by the budgets, so no call
synchronises the host. Equal scores at the k-th place are taken in
ascending tile order (torch.topk leaves that order unspecified).
"""

from __future__ import annotations

import dataclasses
import functools
import math

import numpy as np
import torch

from . import ops
from . import tiling


@dataclasses.dataclass(frozen=True)
class Budget:
    """How many key tiles a query tile keeps in one column block.

    Exactly one field is set: `tiles`, a fixed (possibly fractional) number
    per query tile, or `ratio`, the share of an equal-cost dense budget
    (1 - sparsity; 1 or more keeps the whole block).
    """

    ratio: float | None = None
    tiles: float | None = None

    def __post_init__(self):
        if (self.ratio is None) == (self.tiles is None):
            raise ValueError('a Budget takes a ratio or a tile count, not '
                             'both and not neither')
        value = self.ratio if self.tiles is None else self.tiles
        if value <= 0:
            raise ValueError(f'a Budget keeps at least something, got {self}')

    @classmethod
    def sparsity(cls, percent: float) -> 'Budget':
        """The budget that skips `percent` % of the key tiles."""
        if not 0.0 <= percent < 100.0:
            raise ValueError(f'sparsity is a percentage below 100, got '
                             f'{percent}')
        return cls(ratio=1.0 - percent / 100.0)

    @property
    def keeps_all(self) -> bool:
        return self.ratio is not None and self.ratio >= 1.0

    def per_row(self, real_tokens: int, n_cols: int) -> float:
        """Mean tiles kept by one query tile of a block with `n_cols`
        columns covering `real_tokens` tokens. A ratio is taken of the work
        the block would cost if its tokens filled whole tiles, ceil(real /
        128)^2 pairs, spread over its n_cols rows."""
        if self.tiles is not None:
            return float(self.tiles)
        n_ideal = math.ceil(real_tokens / tiling.TILE_SIZE)
        return self.ratio * n_ideal * n_ideal / n_cols


def split_budget(budget: float, n_cols: int) -> tuple[int, int, float]:
    """A fractional per-row budget as whole tiles: every row keeps k_lo,
    and a share `frac` of the rows keeps k_hi = k_lo + 1 (both within
    [1, n_cols]). `frac` is rounded to 12 decimals, so a budget of 2.3
    yields a fraction that is 0.3 as a double, not 0.29999..., which would
    change which rows get the extra tile."""
    if budget >= n_cols:
        return n_cols, n_cols, 0.0
    k_lo = min(max(1, math.floor(budget)), n_cols)
    frac = round(min(max(budget - k_lo, 0.0), 1.0), 12)
    return k_lo, min(k_lo + 1, n_cols), frac


def _ramp(n_rows: int, frac: float) -> np.ndarray:
    ramp = np.floor(np.arange(n_rows + 1, dtype=np.float64) * frac)
    return ramp[1:] > ramp[:-1]


@functools.lru_cache(maxsize=256)
def _bresenham(n_rows: int, frac: float, device: str) -> torch.Tensor:
    return torch.from_numpy(_ramp(n_rows, frac).astype(np.uint8)).to(device)


def bresenham_extra(n_rows: int, frac: float,
                    device: torch.device | str) -> torch.Tensor:
    """Which rows take the extra tile: [n_rows] uint8, 1 where the fp64
    line floor(r * frac) steps up between r and r + 1, which spreads the
    extras evenly and makes the mean kept count equal the budget. The
    tensor is cached per device and must not be written."""
    return _bresenham(n_rows, float(frac), str(torch.device(device)))


@dataclasses.dataclass(frozen=True)
class ColumnBlock:
    """A range [start, stop) of video key tiles that shares one budget."""

    start: int
    stop: int
    budget: Budget
    real_tokens: int


def column_blocks(layout, generated: Budget,
                  reference: Budget) -> list[ColumnBlock]:
    """The generated (target) block, preceded by the reference block when
    reference spans are tiled."""
    target = ColumnBlock(layout.n_ref_tiles, layout.n_video_tiles, generated,
                         layout.target_tokens)
    if layout.n_ref_tiles == 0:
        return [target]
    return [ColumnBlock(0, layout.n_ref_tiles, reference, layout.ref_tokens),
            target]


def list_width(layout, blocks: list[ColumnBlock]) -> int:
    """Width of the index lists that fits every row without a sync: each
    block's k_hi (its width when it keeps all) plus the global tiles; global
    rows keep every tile."""
    if layout.n_global_tiles:
        return layout.n_tiles
    width = 0
    for block in blocks:
        n_cols = block.stop - block.start
        width += n_cols if block.budget.keeps_all else split_budget(
            block.budget.per_row(block.real_tokens, n_cols), n_cols)[1]
    return max(1, min(width, layout.n_tiles))


@functools.lru_cache(maxsize=64)
def _extra_rows(n_video: int, fracs: tuple[float, ...],
                device: str) -> torch.Tensor:
    rows = [_ramp(n_video, f).astype(np.uint8) for f in fracs]
    return torch.from_numpy(np.stack(rows)).to(device)


def kernel_blocks(layout, blocks: list[ColumnBlock], device):
    """(start, stop, keeps_all, k_lo) per block and the [n_blocks, n_video]
    uint8 Bresenham rows, as the selection kernel takes them."""
    spec, fracs = [], []
    for block in blocks:
        n_cols = block.stop - block.start
        if block.budget.keeps_all:
            spec.append((block.start, block.stop, True, n_cols))
            fracs.append(0.0)
            continue
        k_lo, _, frac = split_budget(
            block.budget.per_row(block.real_tokens, n_cols), n_cols)
        spec.append((block.start, block.stop, False, k_lo))
        fracs.append(frac)
    extra = _extra_rows(layout.n_video_tiles, tuple(fracs),
                        str(torch.device(device))) if blocks else None
    return spec, extra


def select_index(scores: torch.Tensor, layout, blocks: list[ColumnBlock],
                 width: int | None = None):
    """Scores [H', n_video, n_video] -> the ascending kept key tiles of every
    query tile (index [H', n_tiles, width] int32, -1 padded; count
    [H', n_tiles] int32), equal to the reference's
    tile_index_list(block_mask(*select(...)) & kv_ok)."""
    width = list_width(layout, blocks) if width is None else width
    spec, extra = kernel_blocks(layout, blocks, scores.device)
    return ops.select_index(scores, layout.kv_ok, layout.n_tiles, spec, extra,
                            width)


def tile_index_list(mask: torch.Tensor, kv_ok: torch.Tensor,
                    width: int | None = None):
    """A dense block mask [H', n, n] as ascending lists of mask & kv_ok
    (width defaults to n, which needs no sync)."""
    width = mask.shape[-1] if width is None else width
    return ops.mask_to_index(mask, kv_ok, width)


def dense_index(layout, heads: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Full attention as index lists: every query tile keeps every
    non-empty key tile (full_attention_layers / steps, 0% sparsity)."""
    kv = layout.kv_ok
    ids = torch.nonzero(kv).view(-1).to(torch.int32)
    n = layout.n_tiles
    index = ids.view(1, 1, -1).expand(heads, n, -1).contiguous()
    count = torch.full((heads, n), ids.numel(), dtype=torch.int32,
                       device=kv.device)
    return index, count
