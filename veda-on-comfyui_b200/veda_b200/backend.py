"""The reference's backend contract (veda_comfy/backends/base.py) and the
B200 backend that implements it over the sm_100a library.

`Backend.attend(q, k, v, block_mask, layout) -> out` has the reference's
argument meaning (base.py:61-77): q / k / v [N, H', 128] contiguous in tile
order with zero padding slots, block_mask [H', n_tiles, n_tiles] bool with
query tiles as rows, `layout` a tile layout (this package's TileLayout or
the reference's own: only valid_count, kv_ok, n_tiles are read). The output
is [N, H', 128] in q's dtype; padding rows are unspecified.

Errors follow base.py:28-39: `BackendUnavailable` when the backend cannot
run here (message shown to the user), `MissingDependency` when the user can
fix it by building the library. `self_test` is base.py:123-155: the result
must be within `tolerance` x absmax of fp32 masked attention and must not
be the dense result.
"""

from __future__ import annotations

import abc

import torch

from . import _lib
from . import kernels
from . import ops
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
    """fp32 masked softmax attention, the self-test's yardstick
    (core/reference.py:14-36): O(N^2) memory, small problems only."""
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


def selftest_problem(device: torch.device, dtype: torch.dtype, seed: int = 0):
    """The reference's self-test problem (base.py:94-120): text 70 | history
    1x8x16 | audio 40 | target 5x8x8 tiled 4x4x8, 2 heads, x ~ 1.5 N(0,1),
    budgets 2 (generated) / 1 (reference) tiles.

    Returns (q, k, v, block_mask, layout).
    """
    spans = [tiling.TiledSpan(70, (1, 8, 16), tiling.TileShape(1, 8, 16)),
             tiling.TiledSpan(238, (5, 8, 8), tiling.TileShape(4, 4, 8))]
    seq_len = 238 + 320
    layout = tiling.build_tile_layout(spans, seq_len, device)
    generator = torch.Generator().manual_seed(seed)
    heads, dim = 2, 128
    x = torch.randn(3, seq_len, heads, dim, generator=generator) * 1.5
    head_ids = torch.arange(heads, device=device)
    q, k, v = (tiling.gather_tiles(t.to(device=device, dtype=dtype), layout,
                                   head_ids) for t in x)
    scores = torch.randn(heads, layout.n_video_tiles, layout.n_video_tiles,
                         generator=generator).to(device)
    blocks = selection.column_blocks(layout, selection.Budget(tiles=2),
                                     selection.Budget(tiles=1))
    index, count = selection.select_index(scores, layout, blocks)
    mask = mask_from_lists(index, count, layout.n_tiles)
    return q, k, v, mask, layout


def self_test(backend: Backend, device: torch.device,
              dtype: torch.dtype = torch.bfloat16) -> None:
    """Checks `backend` against fp32 masked attention on `device`.

    Raises:
        BackendUnavailable: If the result is wrong, dense, or the kernels
            reported a device-side error.
    """
    if dtype not in backend.dtypes:
        dtype = backend.dtypes[0]
    try:
        q, k, v, mask, layout = selftest_problem(device, dtype)
        out = backend.attend(q, k, v, mask, layout)
        ops.check_status(device)
    except BackendUnavailable:
        raise
    except Exception as error:  # kernels fail in many ways; report, not crash
        raise BackendUnavailable(
            f'{backend.name} failed its self-test: {type(error).__name__}: '
            f'{error}') from error
    real = layout.slot_valid.bool()
    want = reference_attention(q, k, v, mask, layout)[real]
    dense = reference_attention(q, k, v, torch.ones_like(mask) & layout.kv_ok,
                                layout)[real]
    got = out[real].float()
    err = (got - want).abs().max().item()
    gap = (dense - want).abs().max().item()
    if (got - dense).abs().max().item() < 0.5 * gap:
        raise BackendUnavailable(f'{backend.name} ignores the block mask on '
                                 'this device (computes dense attention)')
    limit = backend.tolerance * max(1.0, want.abs().max().item())
    if not err <= limit:
        raise BackendUnavailable(f'{backend.name} gives wrong results on this '
                                 f'device (max error {err:.3g}, allowed '
                                 f'{limit:.3g})')
