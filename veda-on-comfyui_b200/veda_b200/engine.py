"""One Veda attention layer end to end on the GPU (the engine fast path).

The reference engine (core/engine.py:246-326) runs, per head group and head
chunk, about sixty torch launches: gather q/k/v into tile order, pool, bmm
logits, top-k, dense block mask, a host-synchronising index list, quantise
Q, quantise K, cast V, attend, scatter. This fast path does the same call
in five kernels with no host synchronisation:

    [gather V] -> quant_pool (Q, K int8 + TripPool features, one read; packed
                  rows are read through the tile permutation)
               -> tile_logits (predictor; skipped when scores are given)
               -> select (top-k straight into ascending index lists)
               -> sparse_attention (tcgen05; a packed output is written
                  through the permutation)

`full=True` is a full-attention layer or step (full_attention_layers /
full_attention_steps, 0% sparsity): the same attention kernel over every
non-empty key tile. Buffers are reused across calls of the same shape.
"""

from __future__ import annotations

import torch

from . import kernels
from . import ops
from . import selection


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
        self._buffers: dict = {}
        self._dense: dict = {}

    def _dense_lists(self, layout, heads: int):
        key = (id(layout), heads)
        hit = self._dense.get(key)
        if hit is None or hit[0] is not layout:
            index, count = selection.dense_index(layout, heads)
            hit = (layout, index, count)
            self._dense[key] = hit
        return hit[1], hit[2]

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
              proj_k: torch.Tensor | None = None, full: bool = False,
              out: torch.Tensor | None = None,
              tiled: bool | None = None,
              out_multicast: int = 0) -> torch.Tensor:
        """Veda attention of one layer.

        Args:
            q, k, v: [S, H, 128] packed rows, or [N, H, 128] already in tile
                order (N = layout.num_slots, padding rows zero).
            layout: Tile layout of the sequence.
            scores: [H, n_video, n_video] tile scores; when None they are
                computed from `proj_q` / `proj_k` ([H, 384, 128]).
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
            # permutation and the attention epilogue writes the output
            # through it, so only V is gathered into tile order.
            perm = layout.perm
            q_t, k_t = q, k
            v_t = ops.gather_tiles(v, perm,
                                   torch.arange(heads, device=q.device))
        dim = q.shape[-1]
        scale = dim ** -0.5 if self.softmax_scale is None \
            else self.softmax_scale
        need_pool = not full and scores is None
        if need_pool and (proj_q is None or proj_k is None):
            raise ValueError('pass tile scores or both predictor projections')
        quant = ops.quant_pool(q_t, k_t, layout.valid_count,
                               layout.n_video_tiles, scale * kernels.LOG2E,
                               pool=need_pool,
                               out=self._buffers.setdefault(
                                   (tuple(q_t.shape), q_t.device), {}),
                               perm=perm)
        if full:
            index, count = self._dense_lists(layout, heads)
        else:
            if scores is None:
                scores = ops.tile_logits(quant['feats_q'], quant['feats_k'],
                                         proj_q, proj_k)
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
                                    quant['k_i8'], quant['k_scale'], v_t,
                                    index, count, layout.valid_count,
                                    out=out, perm=perm)
