"""One Veda attention layer end to end on the GPU (the engine fast path).

The reference engine (core/engine.py:246-326) runs, per head group and head
chunk, about sixty torch launches: gather q/k/v into tile order, pool, bmm
logits, top-k, dense block mask, a host-synchronising index list, quantise
Q, quantise K, cast V, attend, scatter. This fast path does the same call
in four kernels with no host synchronisation:

    quant_pool (Q, K int8 + TripPool features, one read; packed rows are
                read through the tile permutation, and packed V is copied
                into tile order by the same launch)
    -> tile_logits (predictor; skipped when scores are given)
    -> select (top-k straight into ascending index lists)
    -> sparse_attention (tcgen05; a packed output is written through the
                         permutation)

`full=True` is a full-attention layer or step (full_attention_layers /
full_attention_steps, 0% sparsity): the same attention kernel over every
non-empty key tile. Buffers are reused across calls of the same shape.
"""

from __future__ import annotations

import dataclasses
from collections.abc import Sequence

import torch

from . import kernels
from . import ops
from . import predictor
from . import selection


@dataclasses.dataclass
class HeadGroup:
    """Heads of one layer that share a tile shape (core/plans.py:25-29).

    Attributes:
        layout: The tile layout of the group's shape.
        heads: Indices of the group's heads in q / k / v (host ints).
        scores: [H', n_video, n_video] tile scores of these heads, or None
            to score them with `projections`.
        projections: The group's predictor projections ([H', 384, 128]
            each; e.g. `predictor.LayerProjections` of a stager), or None.
    """

    layout: object
    heads: Sequence[int]
    scores: torch.Tensor | None = None
    projections: predictor.LayerProjections | None = None


class Stats:
    """What the sparse calls selected, accumulated on the device and read
    once at the end of a run (reading per call would synchronise), in the
    reference's terms (core/engine.py:48-107).

    Work is counted in 128 x 128 tile pairs per head: the kept video pairs
    plus the always-dense global rows and columns, against the
    (seq_len / 128)^2 pairs of full attention, so `compute_fraction` is the
    share of full-attention work done. The per-row spread of kept tiles
    (min, mean, max) tells a steady selection from one that swings between
    neighbouring query tiles.
    """

    def __init__(self):
        self.kept = None
        self.video_pairs = 0
        self.work = None
        self.dense_work = 0.0
        self.row_min = None
        self.row_max = None
        self.row_sum = None
        self.rows = 0

    def add_lists(self, count: torch.Tensor, layout) -> None:
        """Adds one selection, given as the kept-tile counts [H', n_tiles]
        the select kernel wrote: a video row's count is its kept video
        tiles plus every non-empty global tile."""
        heads = count.shape[0]
        n_video = layout.n_video_tiles
        per_row = count[:, :n_video] - layout.n_global_ok
        low, high, total = per_row.min(), per_row.max(), per_row.sum()
        self.row_min = low if self.row_min is None else torch.minimum(
            self.row_min, low)
        self.row_max = high if self.row_max is None else torch.maximum(
            self.row_max, high)
        self.row_sum = total if self.row_sum is None else self.row_sum + total
        self.rows += per_row.numel()
        global_pairs = layout.n_global_tiles * (layout.n_tiles + n_video)
        work = total + heads * global_pairs
        self.kept = total if self.kept is None else self.kept + total
        self.work = work if self.work is None else self.work + work
        self.video_pairs += heads * n_video ** 2
        self.dense_work += heads * (layout.seq_len / 128) ** 2

    def kept_fraction(self) -> float | None:
        """Kept share of the video x video tile pairs."""
        if self.kept is None or not self.video_pairs:
            return None
        return float(self.kept) / self.video_pairs

    def per_row(self) -> tuple[int, float, int] | None:
        """(min, mean, max) video key tiles kept per query tile, or None."""
        if self.row_sum is None or not self.rows:
            return None
        return (int(self.row_min), float(self.row_sum) / self.rows,
                int(self.row_max))

    def compute_fraction(self) -> float | None:
        """Share of full-attention work done (all rows, all tokens)."""
        if self.work is None or not self.dense_work:
            return None
        return min(1.0, float(self.work) / self.dense_work)


class VedaAttention:
    """Sparse attention for one pair of budgets on one device.

    Args:
        generated: Budget of the generated (target) video's key tiles.
        reference: Budget of the tiled reference spans' key tiles.
        softmax_scale: Defaults to head_dim ** -0.5.
    """

    def __init__(self, generated: selection.Budget,
                 reference: selection.Budget = selection.Budget(ratio=1.0),
                 softmax_scale: float | None = None):
        self.generated = generated
        self.reference = reference
        self.softmax_scale = softmax_scale
        self.stats = Stats()
        self._buffers: dict = {}
        self._dense: dict = {}
        self._head_ids: dict = {}

    def _dense_lists(self, layout, heads: int):
        key = (id(layout), heads)
        hit = self._dense.get(key)
        if hit is None or hit[0] is not layout:
            index, count = selection.dense_index(layout, heads)
            hit = (layout, index, count)
            self._dense[key] = hit
        return hit[1], hit[2]

    def _ids(self, heads, n_heads: int, device) -> torch.Tensor:
        key = (tuple(int(h) for h in heads), n_heads, device)
        hit = self._head_ids.get(key)
        if hit is None:
            ids = ops.head_ids(list(key[0]), n_heads, device)
            self._head_ids[key] = hit = ids
        return hit

    @torch.no_grad()
    def attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  groups: Sequence[HeadGroup], *, full: bool = False,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """One layer over every head group of its tile plan
        (core/engine.py:282-323): packed q / k / v [S, H, 128] in, packed
        [S, H, 128] out in v's dtype.

        Each group runs its own kernel sequence on the same packed tensors:
        Q and K quantised (and pooled) and V copied into tile order, all
        through its permutation and head ids in one launch, its scores
        selected into lists, and its attention writing its heads of `out`
        through the permutation. No per-group copy of q, k or v is taken
        with torch, nothing synchronises the host, and the selection counts
        feed `self.stats`.
        """
        seq_len, n_heads, dim = q.shape
        device = q.device
        if out is None:
            # every row of the sequence is a tile slot of every layout, and
            # the groups cover every head: all of `out` is written
            out = torch.empty(seq_len, n_heads, dim, dtype=v.dtype,
                              device=device)
        scale = dim ** -0.5 if self.softmax_scale is None \
            else self.softmax_scale
        for group in groups:
            layout = group.layout
            if layout.seq_len != seq_len:
                raise ValueError(f'a layout of {layout.seq_len} rows for a '
                                 f'sequence of {seq_len}')
            ids32 = self._ids(group.heads, n_heads, device)
            perm = layout.perm
            need_pool = not full and group.scores is None
            if need_pool and group.projections is None:
                raise ValueError('a head group needs scores or projections')
            quant = ops.quant_pool(
                q, k, layout.valid_count, layout.n_video_tiles,
                scale * kernels.LOG2E, pool=need_pool,
                out=self._buffers.setdefault(
                    ('group', layout.num_slots, ids32.numel(), device), {}),
                perm=perm, heads=ids32, v=v)
            if full:
                index, count = self._dense_lists(layout, ids32.numel())
            else:
                scores = group.scores
                if scores is None:
                    scores = group.projections.logits(quant['feats_q'],
                                                      quant['feats_k'])
                index, count = self.select(scores, layout)
                self.stats.add_lists(count, layout)
            ops.sparse_attention(quant['q_i8'], quant['q_scale'],
                                 quant['k_i8'], quant['k_scale'],
                                 quant['v_tiled'], index, count,
                                 layout.valid_count, out=out, perm=perm,
                                 heads=ids32)
        return out

    @torch.no_grad()
    def select(self, scores: torch.Tensor, layout):
        """Index lists of one layer from its tile scores."""
        blocks = selection.column_blocks(layout, self.generated,
                                         self.reference)
        return selection.select_index(scores, layout, blocks)

    @torch.no_grad()
    def layer(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              layout, *, scores: torch.Tensor | None = None,
              proj_q: torch.Tensor | None = None,
              proj_k: torch.Tensor | None = None,
              projections: predictor.LayerProjections | None = None,
              full: bool = False,
              out: torch.Tensor | None = None,
              tiled: bool | None = None,
              out_multicast: int = 0) -> torch.Tensor:
        """Veda attention of one layer.

        Args:
            q, k, v: [S, H, 128] packed rows, or [N, H, 128] already in tile
                order (N = layout.num_slots, padding rows zero).
            layout: Tile layout of the sequence.
            scores: [H, n_video, n_video] tile scores; when None they are
                computed by the predictor from `projections` (a layer of a
                `predictor.ProjectionStager`, fp8 storage included) or from
                `proj_q` / `proj_k` ([H, 384, 128] on the device).
            full: Full attention (every non-empty key tile).
            out: Optional output [S or N, H, 128].
            tiled: Whether q / k / v are already in tile order. By default
                they are when they have N rows and either the layout is the
                identity or N differs from the packed length S.
            out_multicast: Head-sharded output (tile-order inputs only):
                the NVSwitch multicast address of `out`'s first element,
                through which the attention kernel writes every row to all
                GPUs bound to the multicast object (see `sharding`).

        Returns:
            Attention output with q's leading shape and v's dtype, in the
            order of the inputs (tile order for tiled inputs).
        """
        heads = q.shape[1]
        if tiled is None and q.shape[0] not in (layout.num_slots,
                                                 layout.seq_len):
            raise ValueError(f'q has {q.shape[0]} rows: expected the '
                             f'layout\'s {layout.seq_len} packed rows or '
                             f'{layout.num_slots} tile slots')
        if tiled is False and q.shape[0] < layout.seq_len:
            raise ValueError(f'packed q has {q.shape[0]} rows, fewer than '
                             f'the layout\'s {layout.seq_len}')
        if tiled is None:
            tiled = q.shape[0] == layout.num_slots and (
                layout.identity or q.shape[0] != layout.seq_len)
        tiled_in = tiled
        perm = None
        if tiled_in:
            q_t, k_t, v_t = q, k, v
        else:
            # Packed rows: the quantisation reads Q and K through the
            # permutation and copies V into tile order in the same launch;
            # the attention writes the output back through it.
            perm = layout.perm
            q_t, k_t, v_t = q, k, None
        dim = q.shape[-1]
        scale = dim ** -0.5 if self.softmax_scale is None \
            else self.softmax_scale
        need_pool = not full and scores is None
        if need_pool and projections is None:
            if proj_q is None or proj_k is None:
                raise ValueError('pass tile scores or the predictor '
                                 'projections')
            projections = predictor.LayerProjections(proj_q, proj_k)
        quant = ops.quant_pool(q_t, k_t, layout.valid_count,
                               layout.n_video_tiles, scale * kernels.LOG2E,
                               pool=need_pool,
                               out=self._buffers.setdefault(
                                   (tuple(q_t.shape), q_t.device), {}),
                               perm=perm, v=None if tiled_in else v)
        if full:
            index, count = self._dense_lists(layout, heads)
        else:
            if scores is None:
                ws = self._buffers.setdefault(('logits', q.device), {})
                need = 2 * layout.n_video_tiles * heads * ops.HEAD_DIM
                if ws.get('w') is None or ws['w'].numel() < need:
                    ws['w'] = torch.empty(need, dtype=torch.float32,
                                          device=q.device)
                scores = projections.logits(quant['feats_q'],
                                            quant['feats_k'], ws['w'])
            index, count = self.select(scores, layout)
        if tiled_in:
            return ops.sparse_attention(
                quant['q_i8'], quant['q_scale'], quant['k_i8'],
                quant['k_scale'], v_t, index, count, layout.valid_count,
                out=out, out_multicast=out_multicast)
        if out_multicast:
            raise ValueError('a multicast output needs tile-order inputs')
        if out is None:
            # every row of the sequence belongs to a tile slot, so the
            # kernel writes all of them: no clearing pass
            out = torch.empty(q.shape[0], heads, dim, dtype=v.dtype,
                              device=q.device)
        return ops.sparse_attention(quant['q_i8'], quant['q_scale'],
                                    quant['k_i8'], quant['k_scale'],
                                    quant['v_tiled'], index, count,
                                    layout.valid_count, out=out, perm=perm)
