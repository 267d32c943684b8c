"""Veda selection rules restated in numpy (test oracle only).

Follows veda_comfy/core/selection.py:
  * Budget.per_row     selection.py:69-73   (tiles, or equal-cost ratio)
  * split_budget       selection.py:81-89   (k_lo, k_hi, frac rounded to 12)
  * bresenham_extra    selection.py:92-106  (fp64 floor ramp)
  * column_blocks      selection.py:119-128 (reference block, then target)
  * select             selection.py:132-180 (kv_ok -> -inf, own tile ->
                       +inf, top-k_hi, keep the first k_lo + extra[row]
                       entries whose value is > -inf)
  * block_mask         selection.py:184-203 (global rows / cols = kv_ok)
  * tile_index_list    selection.py:206-227 (ascending kept tile ids)

Tie order: `torch.topk` leaves the order of equal values unspecified. This
oracle defines it as "lower tile id first" (a stable sort on the value),
which is what the CUDA selection implements, and `boundary_ties` reports
rows where that choice decides membership, so a comparison against the
reference can set them apart.
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np

from . import tiling


@dataclasses.dataclass(frozen=True)
class Budget:
    ratio: float | None = None
    tiles: float | None = None

    @classmethod
    def sparsity(cls, percent: float) -> 'Budget':
        return cls(ratio=1.0 - percent / 100.0)

    @property
    def keeps_all(self) -> bool:
        return self.ratio is not None and self.ratio >= 1.0

    def per_row(self, real_tokens: int, n_cols: int) -> float:
        if self.tiles is not None:
            return float(self.tiles)
        n_ideal = math.ceil(real_tokens / tiling.TILE)
        return self.ratio * n_ideal * n_ideal / n_cols


def split_budget(budget: float, n_cols: int) -> tuple[int, int, float]:
    if budget >= n_cols:
        return n_cols, n_cols, 0.0
    k_lo = min(max(1, math.floor(budget)), n_cols)
    frac = round(min(max(budget - k_lo, 0.0), 1.0), 12)
    return k_lo, min(k_lo + 1, n_cols), frac


def bresenham_extra(n_rows: int, frac: float) -> np.ndarray:
    ramp = np.floor(np.arange(n_rows + 1, dtype=np.float64) * frac)
    return ramp[1:] > ramp[:-1]


@dataclasses.dataclass(frozen=True)
class ColumnBlock:
    start: int
    stop: int
    budget: Budget
    real_tokens: int


def column_blocks(layout: tiling.Layout, generated: Budget,
                  reference: Budget) -> list[ColumnBlock]:
    target = ColumnBlock(layout.n_ref_tiles, layout.n_video_tiles, generated,
                         layout.target_tokens)
    if layout.n_ref_tiles == 0:
        return [target]
    return [ColumnBlock(0, layout.n_ref_tiles, reference, layout.ref_tokens),
            target]


def _block_scores(scores, layout, block):
    n_video = layout.n_video_tiles
    n_cols = block.stop - block.start
    s = scores[:, :, block.start:block.stop].astype(np.float32).copy()
    s[:, :, ~layout.kv_ok[block.start:block.stop]] = -np.inf
    rows = np.arange(n_video)
    own = (rows >= block.start) & (rows < block.stop)
    s[:, rows[own], rows[own] - block.start] = np.inf
    del n_cols
    return s


def select_keep(scores: np.ndarray, layout: tiling.Layout,
                blocks: list[ColumnBlock]) -> np.ndarray:
    """[H, n_video, n_video] scores -> [H, n_video, n_video] bool of the
    kept video key tiles (the video quadrant of the block mask)."""
    heads, n_video = scores.shape[0], layout.n_video_tiles
    keep = np.zeros((heads, n_video, n_video), dtype=bool)
    for block in blocks:
        n_cols = block.stop - block.start
        if block.budget.keeps_all:
            keep[:, :, block.start:block.stop] = \
                layout.kv_ok[block.start:block.stop]
            continue
        s = _block_scores(scores, layout, block)
        k_lo, _, frac = split_budget(
            block.budget.per_row(block.real_tokens, n_cols), n_cols)
        allowed = k_lo + bresenham_extra(n_video, frac).astype(np.int64)
        # stable sort on the negated value: equal values keep ascending id
        order = np.argsort(-s, axis=-1, kind='stable')
        vals = np.take_along_axis(s, order, axis=-1)
        rank_ok = np.arange(n_cols)[None, None, :] < allowed[None, :, None]
        chosen = rank_ok & (vals > -np.inf)
        sub = np.zeros_like(chosen)
        np.put_along_axis(sub, order, chosen, axis=-1)
        keep[:, :, block.start:block.stop] = sub
    return keep


def boundary_ties(scores: np.ndarray, layout: tiling.Layout,
                  blocks: list[ColumnBlock]) -> np.ndarray:
    """[H, n_video] bool: rows whose kept set depends on the tie order."""
    heads, n_video = scores.shape[0], layout.n_video_tiles
    ties = np.zeros((heads, n_video), dtype=bool)
    for block in blocks:
        n_cols = block.stop - block.start
        if block.budget.keeps_all:
            continue
        s = _block_scores(scores, layout, block)
        k_lo, _, frac = split_budget(
            block.budget.per_row(block.real_tokens, n_cols), n_cols)
        allowed = k_lo + bresenham_extra(n_video, frac).astype(np.int64)
        vals = -np.sort(-s, axis=-1, kind='stable')
        for r in range(n_video):
            kk = allowed[r]
            if kk >= n_cols:
                continue
            last, nxt = vals[:, r, kk - 1], vals[:, r, kk]
            ties[:, r] |= (last == nxt) & (last > -np.inf)
    return ties


def block_mask(keep: np.ndarray, layout: tiling.Layout) -> np.ndarray:
    heads = keep.shape[0]
    n, n_video = layout.n_tiles, layout.n_video_tiles
    mask = np.zeros((heads, n, n), dtype=bool)
    mask[:, :n_video, :n_video] = keep
    mask[:, :, n_video:] = layout.kv_ok[n_video:]
    mask[:, n_video:, :] = layout.kv_ok
    return mask


def tile_index_list(mask: np.ndarray, width: int | None = None):
    """mask [H, n, n] -> (index [H, n, width] int32 ascending, -1 past the
    count; count [H, n] int32). width defaults to the widest row."""
    count = mask.sum(-1).astype(np.int32)
    widest = int(count.max()) if count.size else 0
    width = widest if width is None else width
    if width < widest:
        raise ValueError(f'width {width} < widest row {widest}')
    order = np.argsort(~mask, axis=-1, kind='stable')[..., :width]
    index = order.astype(np.int32)
    live = np.arange(width)[None, None, :] < count[..., None]
    index[~live] = -1
    return index, count


def index_lists(scores, layout, blocks, width=None):
    """The whole selection: scores -> ascending kept key tiles per query
    tile (video and global rows) and their counts."""
    mask = block_mask(select_keep(scores, layout, blocks), layout)
    return tile_index_list(mask & layout.kv_ok[None, None, :], width)


def max_width(layout: tiling.Layout, blocks: list[ColumnBlock]) -> int:
    """A row-count bound that needs no device sync: every block's k_hi (or
    its whole width when it keeps all), plus the global tiles; global rows
    keep every tile."""
    width = layout.n_global_tiles
    for block in blocks:
        n_cols = block.stop - block.start
        if block.budget.keeps_all:
            width += n_cols
        else:
            width += split_budget(
                block.budget.per_row(block.real_tokens, n_cols), n_cols)[1]
    if layout.n_global_tiles:
        width = layout.n_tiles
    return min(width, layout.n_tiles)
