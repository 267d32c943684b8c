"""The kernel package API of the reference (`veda_comfy.kernels.sage.
sparse_int8`: `quantize`, `key_blocks`, `attend`, `available`) over the
sm_100a library.

`attend` takes the same arguments and gives the same result contract as
sparse_int8.py:312-362: tile-ordered [N, H, 128] 16-bit q / k / v, index
[H, N/128, W] ascending kept tile ids with `count` of them real, the tiles'
valid counts, and an optional softmax scale; it returns [N, H, 128] in v's
dtype. Two differences, both internal: Q and K are quantised in one fused
pass into head-major int8 (the layout the TMA tile loads read), and the
kernel walks 128-row key tiles with K's two 64-row scales applied per
column half, so no `key_blocks` expansion is needed (it is kept for API
parity).
"""

from __future__ import annotations

import torch

from . import _lib
from . import ops

TILE = ops.TILE
KEY_BLOCK = ops.KEY_BLOCK
LOG2E = 1.4426950408889634


def quantize(x: torch.Tensor, block: int, pre_scale: float = 1.0):
    """[N, H, D] -> (int8 [H, N, D] head-major, fp32 [H, N // block])."""
    return ops.quantize(x, block, pre_scale)


def key_blocks(index: torch.Tensor, count: torch.Tensor,
               valid_count: torch.Tensor, block: int = KEY_BLOCK):
    """Kept 128-row tiles -> kept `block`-row key blocks and their valid
    row counts (the reference's host-side expansion)."""
    sub = TILE // block
    blocks = (index.to(torch.int32) * sub)[..., None] + torch.arange(
        sub, device=index.device, dtype=torch.int32)
    offsets = torch.arange(sub, device=valid_count.device) * block
    valid = (valid_count[:, None] - offsets).clamp_(0, block)
    return (blocks.flatten(-2).contiguous(), (count * sub).contiguous(),
            valid.flatten().to(torch.int32).contiguous())


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
           index: torch.Tensor, count: torch.Tensor,
           valid_count: torch.Tensor,
           softmax_scale: float | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Block-sparse INT8 attention on tile-ordered tensors.

    Args:
        q, k, v: [N, H, 128], 16-bit, N a multiple of 128; rows and heads
            16-byte aligned, the head dim contiguous.
        index: [H, N // 128, W] int32 kept key tiles per query tile,
            ascending; entries past `count` are ignored.
        count: [H, N // 128] int32.
        valid_count: [n_tiles] int32 real rows per tile (a prefix).
        softmax_scale: defaults to 128 ** -0.5.

    Returns:
        [N, H, 128] in v's dtype (q's dtype when they agree).
    """
    dim = q.shape[-1]
    scale = dim ** -0.5 if softmax_scale is None else softmax_scale
    if v.dtype != q.dtype:
        v = v.to(q.dtype)
    quant = ops.quant_pool(q, k, valid_count, 0, scale * LOG2E, pool=False)
    return ops.sparse_attention(quant['q_i8'], quant['q_scale'],
                                quant['k_i8'], quant['k_scale'], v, index,
                                count, valid_count, out=out)


def available() -> bool:
    """Whether the library is built and the current device is sm_100."""
    try:
        lib = _lib.load()
    except _lib.VedaError:
        return False
    return (torch.cuda.is_available()
            and bool(lib.veda_device_supported(torch.cuda.current_device())))
