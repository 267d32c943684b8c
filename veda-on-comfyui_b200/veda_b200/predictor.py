"""Veda predictor scoring on the GPU: pooled tile features, tile logits,
and the per-layer staging of the predictor's projections.

Arithmetic of the reference's core/predictor.py: TripPool features
[mean | max | min] over the real rows of every video tile (:20-60), and
tile logits q_hat k_hat^T / sqrt(D) with x_hat = F @ P[h] + F[:, :D]
(:63-80), all fp32. In the engine the pooling runs inside the Q / K
quantisation pass (ops.quant_pool reads Q and K once for both).

Projections. A bundle holds, per DiT layer, [H, 3D, D] projections for q
and k (core/bundle.py:132-189). The reference keeps them on the host in
bf16 (fp8 bundles are dequantised at load) and copies one layer's pair to
the device when that layer runs (core/engine.py:213-227), so the copy sits
in front of the layer's scoring. `ProjectionStager` keeps the host copies
pinned in the bundle's own storage type, fp8 included, and copies the next
layer's pair on a side stream while the current layer computes; fp8 pairs
cross PCIe at half the bytes of bf16 and are dequantised inside the
projection kernel, to the same values the reference's loader produces.
"""

from __future__ import annotations

import torch

from . import ops


def pool_video_tiles(x: torch.Tensor, layout) -> torch.Tensor:
    """[N, H', D] tile-ordered -> [H', n_video_tiles, 3D] fp32 features;
    exactly 0 for empty tiles (the standalone form of the pooling the
    quantisation pass does)."""
    feats = ops.quant_pool(x, x, layout.valid_count, layout.n_video_tiles,
                           1.0, pool=True)
    return feats['feats_q']


def tile_logits(feats_q: torch.Tensor, feats_k: torch.Tensor,
                proj_q: torch.Tensor, proj_k: torch.Tensor,
                workspace: torch.Tensor | None = None,
                scale_q: torch.Tensor | None = None,
                scale_k: torch.Tensor | None = None) -> torch.Tensor:
    """[H', n_q, 3D] x [H', n_k, 3D] features, [H', 3D, D] projections
    (bf16 / fp16 / fp32, or fp8 with per-head scales) -> [H', n_q, n_k]
    fp32 logits."""
    return ops.tile_logits(feats_q, feats_k, proj_q, proj_k, workspace,
                           scale_q, scale_k)


class LayerProjections:
    """One layer's projections on the device: proj_q, proj_k [H, 3D, D] and,
    for fp8 storage, their per-head scales (else None)."""

    __slots__ = ('proj_q', 'proj_k', 'scale_q', 'scale_k')

    def __init__(self, proj_q, proj_k, scale_q=None, scale_k=None):
        self.proj_q, self.proj_k = proj_q, proj_k
        self.scale_q, self.scale_k = scale_q, scale_k

    def logits(self, feats_q: torch.Tensor, feats_k: torch.Tensor,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
        return ops.tile_logits(feats_q, feats_k, self.proj_q, self.proj_k,
                               workspace, self.scale_q, self.scale_k)


class ProjectionStager:
    """Host-resident per-layer projections, copied to the device one layer
    ahead of use.

    Args:
        proj_q, proj_k: Per layer [H, 3D, D] host tensors, all of one dtype
            (bf16, fp16, fp32 or float8_e4m3fn).
        device: The CUDA device the layers run on.
        scale_q, scale_k: Per layer [H] fp32 scales, required for fp8.

    `get(layer)` returns the layer's LayerProjections, valid on the current
    stream, and starts copying layer + 1 into the other of two device slots.
    The copy of a slot waits until every kernel enqueued on the current
    stream before the `get` call that frees it has run, so the device
    buffers are never overwritten while a queued layer still reads them.
    """

    def __init__(self, proj_q: list[torch.Tensor], proj_k: list[torch.Tensor],
                 device: torch.device, scale_q: list[torch.Tensor] | None = None,
                 scale_k: list[torch.Tensor] | None = None):
        if len(proj_q) != len(proj_k) or not proj_q:
            raise ValueError('need the same, non-zero number of q and k '
                             'projections')
        dtype = proj_q[0].dtype
        if any(t.dtype != dtype for t in proj_q + proj_k):
            raise ValueError('all projections must share one storage dtype')
        self.fp8 = dtype == torch.float8_e4m3fn
        if self.fp8 and (scale_q is None or scale_k is None):
            raise ValueError('fp8 projections need per-head scales')
        self.device = torch.device(device)
        self.num_layers = len(proj_q)
        pin = torch.cuda.is_available()
        self._host = [(q.contiguous().pin_memory() if pin else q.contiguous(),
                       k.contiguous().pin_memory() if pin else k.contiguous())
                      for q, k in zip(proj_q, proj_k)]
        self._scales = None
        if self.fp8:
            self._scales = [(sq.float().contiguous(), sk.float().contiguous())
                            for sq, sk in zip(scale_q, scale_k)]
        shape = tuple(proj_q[0].shape)
        heads = shape[0]
        self._slots = [
            LayerProjections(
                torch.empty(shape, dtype=dtype, device=self.device),
                torch.empty(shape, dtype=dtype, device=self.device),
                torch.empty(heads, dtype=torch.float32, device=self.device)
                if self.fp8 else None,
                torch.empty(heads, dtype=torch.float32, device=self.device)
                if self.fp8 else None)
            for _ in range(2)]
        self._layer_in = [-1, -1]      # layer whose copy was issued per slot
        self._ready = [None, None]     # event: that copy finished
        self._stream = torch.cuda.Stream(self.device)

    @property
    def bytes_per_layer(self) -> int:
        q, k = self._host[0]
        return 2 * q.numel() * q.element_size()

    def _copy(self, layer: int) -> None:
        slot = layer % 2
        if self._layer_in[slot] == layer:
            return
        # what the current stream has queued so far may still read the slot
        freed = torch.cuda.current_stream(self.device).record_event()
        with torch.cuda.stream(self._stream):
            self._stream.wait_event(freed)
            dst = self._slots[slot]
            q, k = self._host[layer]
            dst.proj_q.copy_(q, non_blocking=True)
            dst.proj_k.copy_(k, non_blocking=True)
            if self.fp8:
                sq, sk = self._scales[layer]
                dst.scale_q.copy_(sq, non_blocking=True)
                dst.scale_k.copy_(sk, non_blocking=True)
            self._ready[slot] = self._stream.record_event()
        self._layer_in[slot] = layer

    def get(self, layer: int) -> LayerProjections:
        """Layer `layer`'s projections for kernels enqueued on the current
        stream from now on; the next layer's copy starts behind them."""
        if not 0 <= layer < self.num_layers:
            raise IndexError(f'layer {layer} of {self.num_layers}')
        self._copy(layer)
        torch.cuda.current_stream(self.device).wait_event(
            self._ready[layer % 2])
        if layer + 1 < self.num_layers:
            self._copy(layer + 1)
        return self._slots[layer % 2]


def quantize_fp8(proj: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[H, 3D, D] -> (float8_e4m3fn weights, [H] fp32 scales) with one amax
    scale per head (amax / 448), the storage fp8 bundles use."""
    amax = proj.float().abs().amax(dim=(1, 2)).clamp(min=1e-12)
    scale = amax / 448.0
    q = (proj.float() / scale.view(-1, 1, 1)).to(torch.float8_e4m3fn)
    return q, scale
