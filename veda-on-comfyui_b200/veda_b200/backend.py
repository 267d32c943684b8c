"""The backend interface of the reference (veda_comfy/backends/base.py) and
the B200 backend behind it.

A backend takes one head group of one layer in tile order and returns its
attention output: `attend(q, k, v, block_mask, layout)` with q / k / v
[N, H', 128] (padding slots zero), block_mask [H', n_tiles, n_tiles] bool
(row = query tile) and a tile layout, of which only valid_count, kv_ok and
n_tiles are used (this package's TileLayout or the reference's own). The
result is [N, H', 128] in q's dtype; rows of padding slots carry no
meaning (base.py:61-77).

Two error types tell the user what happened (base.py:28-39):
`BackendUnavailable` means this machine cannot run the backend, and
`MissingDependency` that the user can fix it (here: build the library).

The reference validates a backend with its own `base.self_test` before the
first call; integration/b200_int8.py is the module that plugs this backend
into the reference's registry, and the GPU tests run that self-test on it.
"""

from __future__ import annotations

import abc

import torch

from . import _lib
from . import kernels
from . import selection
from . import tiling


class BackendUnavailable(RuntimeError):
    """The backend cannot run here; the message is shown to the user."""


class MissingDependency(BackendUnavailable):
    """Something the backend needs is missing and the user can fix it; the
    message is the fix."""


class Backend(abc.ABC):
    """Block-sparse attention on tile-ordered tensors (base.py:41-91)."""

    name: str = 'backend'
    display: str = 'backend'
    dtypes: tuple[torch.dtype, ...] = (torch.bfloat16, torch.float16)
    tolerance: float = 0.02

    @abc.abstractmethod
    def attend(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               block_mask: torch.Tensor, layout) -> torch.Tensor:
        """Block-sparse attention; see the module docstring."""

    def warmup_note(self) -> str | None:
        return None

    def explain_failure(self, error: BaseException) -> str | None:
        del error
        return None


class B200Int8Backend(Backend):
    """INT8 QK^T / 16-bit PV block-sparse attention on tcgen05 tensor cores.

    Same arithmetic contract as the reference's triton-int8 backend
    (backends/triton_int8.py:36-55): Q per 128 rows and K per 64 rows INT8
    with fp32 scales and the softmax scale folded into Q; P rounded to V's
    16-bit type (bf16 for bf16 inputs, where the reference casts V and P to
    fp16). Tolerance 0.05 of absmax, the reference's figure for this format.
    """

    name = 'b200-int8'
    display = 'B200 INT8 (tcgen05)'
    dtypes = (torch.bfloat16, torch.float16)
    tolerance = 0.05

    def attend(self, q, k, v, block_mask, layout):
        with torch.no_grad():
            index, count = selection.tile_index_list(block_mask, layout.kv_ok)
            return kernels.attend(q, k, v, index, count, layout.valid_count)

    def explain_failure(self, error: BaseException) -> str | None:
        if isinstance(error, _lib.LibraryMissing):
            return ('build the B200 kernels once: '
                    'python -m veda_b200.build (needs CUDA 12.8+ nvcc)')
        return None


def create(device: torch.device | None = None) -> Backend:
    """The B200 backend for `device` (default: the current CUDA device).

    Raises:
        MissingDependency: libveda_b200.so has not been built.
        BackendUnavailable: no CUDA device, or it is not an sm_100 GPU.
    """
    if not torch.cuda.is_available():
        raise BackendUnavailable('b200-int8 needs a CUDA GPU')
    device = torch.device('cuda', torch.cuda.current_device()) \
        if device is None else torch.device(device)
    try:
        lib = _lib.load()
    except _lib.LibraryMissing as error:
        raise MissingDependency(
            f'{error}. Build it with: python -m veda_b200.build') from error
    index = device.index if device.index is not None else \
        torch.cuda.current_device()
    if not lib.veda_device_supported(index):
        cc = torch.cuda.get_device_capability(index)
        raise BackendUnavailable(
            f'b200-int8 needs an sm_100 GPU (B200 / GB200); cuda:{index} is '
            f'sm_{cc[0]}{cc[1]}')
    return B200Int8Backend()


def reference_attention(q, k, v, block_mask, layout) -> torch.Tensor:
    """fp32 masked softmax attention over the kept tiles, the yardstick of
    core/reference.py:14-36: O(N^2) memory, small problems only."""
    tile = tiling.TILE_SIZE
    scale = q.shape[-1] ** -0.5
    allowed = block_mask.repeat_interleave(tile, 1).repeat_interleave(tile, 2)
    allowed = allowed & layout.slot_valid.bool()[None, None, :]
    scores = torch.einsum('qhd,khd->hqk', q.float(), k.float()) * scale
    scores = scores.masked_fill(~allowed, float('-inf'))
    probs = torch.softmax(scores, dim=-1).nan_to_num(0.0)
    out = torch.einsum('hqk,khd->qhd', probs, v.float())
    return out * layout.slot_valid.to(out.dtype)[:, None, None]


def mask_from_lists(index: torch.Tensor, count: torch.Tensor,
                    n_tiles: int) -> torch.Tensor:
    """Index lists [H, n, W] (+ count) -> dense block mask [H, n, n_tiles]."""
    heads, n, width = index.shape
    live = torch.arange(width, device=index.device)[None, None, :] < \
        count[..., None]
    cols = torch.where(live, index.long(), n_tiles)
    mask = torch.zeros(heads, n, n_tiles + 1, dtype=torch.bool,
                       device=index.device)
    mask.scatter_(2, cols, True)
    return mask[..., :n_tiles].contiguous()
