"""Torch-facing wrappers of the C ABI: device tensors in, device tensors out,
launched on the current CUDA stream, no synchronisation.

Every op refuses CPU tensors and non-sm_100 devices; there is no fallback
path. Device-side errors accumulate in a per-device int32 status word that
`check_status` reads (it synchronises, so the hot path never calls it).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

TILE = 128
HEAD_DIM = 128
KEY_BLOCK = 64

_DTYPES = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16,
           torch.float32: _lib.F32}
_status_words: dict[int, torch.Tensor] = {}
_supported: dict[int, bool] = {}


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_device(*tensors: torch.Tensor) -> torch.device:
    """The common CUDA device of `tensors`; raises unless it is sm_100."""
    device = tensors[0].device
    for t in tensors:
        if t.device != device:
            raise ValueError(f'tensors on {t.device} and {device}')
    if device.type != 'cuda':
        raise _lib.VedaError(_lib.ERR_UNSUPPORTED,
                             f'veda_b200 runs on CUDA tensors only, got '
                             f'{device}')
    index = device.index if device.index is not None else \
        torch.cuda.current_device()
    if index not in _supported:
        _supported[index] = bool(_lib.load().veda_device_supported(index))
    if not _supported[index]:
        raise _lib.VedaError(_lib.ERR_UNSUPPORTED,
                             f'cuda:{index} is not an sm_100 GPU')
    return torch.device('cuda', index)


def _call(device: torch.device, name: str, *args) -> None:
    """Runs a C-ABI entry point with `device` current."""
    if torch.cuda.current_device() == device.index:
        _lib.call(name, *args)
    else:
        with torch.cuda.device(device):
            _lib.call(name, *args)


def status_word(device: torch.device) -> torch.Tensor:
    """The device's int32 status word (created zeroed on first use)."""
    index = device.index if device.index is not None else \
        torch.cuda.current_device()
    word = _status_words.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=device)
        _status_words[index] = word
    return word


def check_status(device: torch.device, clear: bool = True) -> None:
    """Synchronises and raises DeviceStatusError if a kernel reported one."""
    word = status_word(device)
    value = int(word.item())
    if clear and value:
        word.zero_()
    if value:
        raise _lib.DeviceStatusError(
            value, f'device status {value:#x}: {_lib.describe_status(value)}')


def _check_rows(x: torch.Tensor, name: str) -> None:
    if x.dim() != 3 or x.shape[-1] != HEAD_DIM:
        raise ValueError(f'{name} must be [slots, heads, 128], got '
                         f'{tuple(x.shape)}')
    if x.stride(-1) != 1:
        raise ValueError(f'{name} must be contiguous along the head dim')
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f'{name} must be bf16 or fp16, got {x.dtype}')


def quantize(x: torch.Tensor, block: int, pre_scale: float = 1.0):
    """[N, H, 128] 16-bit -> (int8 [H, N, 128], fp32 scales [H, N // block]).

    Arithmetic of sparse_int8.quantize; the int8 tensor is head-major, the
    layout the attention kernel's TMA tile loads read.
    """
    _check_rows(x, 'x')
    device = require_device(x)
    n, heads, _ = x.shape
    out = torch.empty(heads, n, HEAD_DIM, dtype=torch.int8, device=device)
    scale = torch.empty(heads, n // block, dtype=torch.float32, device=device)
    _call(device, 'veda_quantize', _ptr(x), _DTYPES[x.dtype], x.stride(0),
              x.stride(1), n, heads, HEAD_DIM, block, ctypes.c_float(pre_scale),
              _ptr(out), _ptr(scale), _stream(device))
    return out, scale


def head_ids(heads, n_heads: int, device: torch.device) -> torch.Tensor:
    """A head group's ids as the kernels take them: [H'] int32 on `device`,
    each checked (on the host, before any launch) to be a head of an input
    with `n_heads` heads."""
    ids = torch.as_tensor(heads).reshape(-1)
    if ids.device.type != 'cpu':
        ids = ids.cpu()
    if ids.numel() == 0 or int(ids.min()) < 0 or int(ids.max()) >= n_heads:
        raise ValueError(f'head ids must lie in [0, {n_heads})')
    return ids.to(device=device, dtype=torch.int32)


def quant_pool(q: torch.Tensor, k: torch.Tensor, valid_count: torch.Tensor,
               n_video_tiles: int, q_pre_scale: float, pool: bool = True,
               out: dict | None = None,
               perm: torch.Tensor | None = None,
               heads: torch.Tensor | None = None,
               v: torch.Tensor | None = None) -> dict:
    """Fused INT8 quantisation of Q (per 128 rows) and K (per 64 rows) and,
    if `pool`, the [mean | max | min] features of the video tiles.

    perm: packed input. q and k are then [S, H, 128] in sequence order and
    tile slot i reads row perm[i] (< 0: padding, zeros): the gather into
    tile order happens in the same read.
    heads: with `perm`, one head group: [H'] int32 device ids (see
    `head_ids`); output head h holds input head heads[h].
    v: with `perm`, packed V [S, H, 128] of q's dtype, copied through the
    same permutation and head ids into `v_tiled` ([slots, H', 128], tile
    order) by the same launch: the V operand of the attention.

    Returns dict(q_i8, q_scale, k_i8, k_scale, feats_q, feats_k[, v_tiled])
    in tile order; buffers in `out` with those names are reused.
    """
    _check_rows(q, 'q')
    _check_rows(k, 'k')
    if q.shape != k.shape or q.stride() != k.stride() or q.dtype != k.dtype:
        raise ValueError('q and k must share shape, strides and dtype')
    device = require_device(q, k, valid_count)
    seq_len, n_in, _ = q.shape
    head_map = heads
    heads = n_in
    if head_map is not None:
        if perm is None:
            raise ValueError('a head group needs packed inputs (perm)')
        if head_map.dtype != torch.int32 or head_map.device != device:
            raise ValueError('heads must be int32 ids on the inputs\' device')
        heads = head_map.numel()
    if perm is not None:
        perm = perm.to(device=device, dtype=torch.int64).contiguous()
    n = seq_len if perm is None else perm.numel()
    n_tiles = n // TILE
    out = {} if out is None else out

    def buf(name, shape, dtype):
        t = out.get(name)
        if t is None or t.shape != shape or t.dtype != dtype:
            t = torch.empty(shape, dtype=dtype, device=device)
            out[name] = t
        return t

    q_i8 = buf('q_i8', (heads, n, HEAD_DIM), torch.int8)
    k_i8 = buf('k_i8', (heads, n, HEAD_DIM), torch.int8)
    q_scale = buf('q_scale', (heads, n_tiles), torch.float32)
    k_scale = buf('k_scale', (heads, 2 * n_tiles), torch.float32)
    feats_q = feats_k = None
    if pool and n_video_tiles > 0:
        feats_q = buf('feats_q', (heads, n_video_tiles, 3 * HEAD_DIM),
                      torch.float32)
        feats_k = buf('feats_k', (heads, n_video_tiles, 3 * HEAD_DIM),
                      torch.float32)
    v_tiled = None
    if v is not None:
        if perm is None:
            raise ValueError('a V copy needs packed inputs (perm)')
        _check_rows(v, 'v')
        if v.dtype != q.dtype or v.shape[0] != seq_len or \
                v.device != device:
            raise ValueError('v must be packed like q (rows, dtype, device)')
        v_tiled = buf('v_tiled', (n, heads, HEAD_DIM), v.dtype)
    valid = valid_count.to(torch.int32)
    tail = (_ptr(valid), n_video_tiles, ctypes.c_float(q_pre_scale),
            _ptr(q_i8), _ptr(q_scale), _ptr(k_i8), _ptr(k_scale),
            _ptr(feats_q), _ptr(feats_k), _stream(device))
    if perm is None:
        _call(device, 'veda_quant_pool', _ptr(q), _ptr(k), _DTYPES[q.dtype],
              q.stride(0), q.stride(1), n, heads, *tail)
    else:
        _call(device, 'veda_quant_pool_packed', _ptr(q), _ptr(k),
              _DTYPES[q.dtype], q.stride(0), q.stride(1), seq_len, _ptr(perm),
              n, heads, *tail[:-1], _ptr(v),
              v.stride(0) if v is not None else 0,
              v.stride(1) if v is not None else 0, _ptr(v_tiled),
              _ptr(head_map), tail[-1])
    out['feats_q'], out['feats_k'] = feats_q, feats_k
    if v_tiled is not None:
        out['v_tiled'] = v_tiled
    return out


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """`t`, or a copy of it that starts 16-byte aligned (a contiguous view
    can start at any element; the logits kernels read 16-byte vectors)."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def tile_logits(feats_q: torch.Tensor, feats_k: torch.Tensor,
                proj_q: torch.Tensor, proj_k: torch.Tensor,
                workspace: torch.Tensor | None = None,
                scale_q: torch.Tensor | None = None,
                scale_k: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """[H, n_q, 384] x [H, n_k, 384] with [H, 384, 128] projections ->
    [H, n_q, n_k] fp32 logits.

    Projections are bf16, fp16, fp32, or fp8 (float8_e4m3fn) with per-head
    fp32 scales `scale_q` / `scale_k` [H], used as bf16(w * scale) like the
    reference's bundle loader stores them.
    """
    device = require_device(feats_q, feats_k, proj_q, proj_k)
    heads, n_q, _ = feats_q.shape
    n_k = feats_k.shape[1]
    feats_q = _aligned(feats_q.float().contiguous())
    feats_k = _aligned(feats_k.float().contiguous())
    if proj_q.dtype != proj_k.dtype:
        raise ValueError('proj_q and proj_k must share a dtype')
    proj_q, proj_k = _aligned(proj_q.contiguous()), _aligned(proj_k.contiguous())
    fp8 = proj_q.dtype == torch.float8_e4m3fn
    if fp8:
        if scale_q is None or scale_k is None:
            raise ValueError('fp8 projections need per-head scales')
        scale_q = scale_q.to(device=device, dtype=torch.float32).contiguous()
        scale_k = scale_k.to(device=device, dtype=torch.float32).contiguous()
        dtype = _lib.FP8_E4M3
    else:
        dtype = _DTYPES[proj_q.dtype]
        scale_q = scale_k = None
    need = (n_q + n_k) * heads * HEAD_DIM
    if workspace is None or workspace.numel() < need or \
            workspace.data_ptr() % 16:
        workspace = torch.empty(need, dtype=torch.float32, device=device)
    logits = out if out is not None else torch.empty(
        heads, n_q, n_k, dtype=torch.float32, device=device)
    _call(device, 'veda_tile_logits_scaled', _ptr(feats_q), _ptr(feats_k),
          _ptr(proj_q), _ptr(proj_k), dtype, _ptr(scale_q), _ptr(scale_k),
          heads, n_q, n_k, _ptr(workspace), _ptr(logits), _stream(device))
    return logits


def select_index(scores: torch.Tensor, kv_ok: torch.Tensor, n_tiles: int,
                 blocks: list[tuple[int, int, bool, int]],
                 extra: torch.Tensor | None, width: int):
    """Top-k selection into ascending lists.

    blocks: (start, stop, keeps_all, k_lo) per column block; extra: uint8
    [n_blocks, n_video] Bresenham rows. Returns (index [H, n_tiles, width]
    int32, -1 padded; count [H, n_tiles] int32).
    """
    device = require_device(scores, kv_ok)
    heads, n_video = scores.shape[0], scores.shape[1]
    if scores.dtype != torch.float32 or scores.stride(-1) != 1:
        scores = scores.float().contiguous()
    kv = kv_ok.to(torch.uint8).contiguous()
    index = torch.empty(heads, n_tiles, width, dtype=torch.int32, device=device)
    count = torch.empty(heads, n_tiles, dtype=torch.int32, device=device)
    arr = (_lib.ColumnBlock * max(1, len(blocks)))(
        *[_lib.ColumnBlock(s, e, int(a), k) for s, e, a, k in blocks])
    _call(device, 'veda_select', _ptr(scores), scores.stride(0), scores.stride(1),
              heads, n_video, n_tiles, _ptr(kv), len(blocks), arr,
              _ptr(extra), width, _ptr(index), _ptr(count),
              _ptr(status_word(device)), _stream(device))
    return index, count


def mask_to_index(mask: torch.Tensor, kv_ok: torch.Tensor, width: int):
    """Dense block mask [H, n, n] -> ascending lists of mask & kv_ok."""
    device = require_device(mask, kv_ok)
    heads, n_tiles = mask.shape[0], mask.shape[1]
    m = mask.contiguous()
    if m.dtype == torch.bool:
        m = m.view(torch.uint8)
    kv = kv_ok.to(torch.uint8).contiguous()
    index = torch.empty(heads, n_tiles, width, dtype=torch.int32, device=device)
    count = torch.empty(heads, n_tiles, dtype=torch.int32, device=device)
    _call(device, 'veda_mask_to_index', _ptr(m), _ptr(kv), heads, n_tiles, width,
              _ptr(index), _ptr(count), _ptr(status_word(device)),
              _stream(device))
    return index, count


def sparse_attention(q_i8, q_scale, k_i8, k_scale, v, index, count,
                     valid_count, out: torch.Tensor | None = None,
                     out_multicast: int = 0,
                     perm: torch.Tensor | None = None,
                     heads: torch.Tensor | None = None):
    """INT8 block-sparse attention. v [N, H, 128] 16-bit in tile order;
    returns out [N, H, 128] of v's dtype (or writes `out`, any row / head
    strides).

    out_multicast: the NVSwitch multicast address of `out`'s first element
    (head sharding): rows are stored through it to every GPU bound to the
    multicast object, instead of to `out` alone.
    perm: packed output. `out` ([S, H, 128], required) receives row `slot`
    of the result at row perm[slot]; padding slots (perm < 0) are dropped:
    the scatter back to sequence order happens in the kernel's epilogue.
    heads: with `perm`, one head group: head h of v / the lists is written to
    head heads[h] of `out` ([H'] int32 device ids, see `head_ids`).
    """
    _check_rows(v, 'v')
    device = require_device(q_i8, k_i8, v, index, count, valid_count)
    head_map = heads
    n, heads, _ = v.shape
    n_tiles = n // TILE
    if head_map is not None and perm is None:
        raise ValueError('a head group needs a packed output (perm)')
    if perm is not None:
        if out is None or out_multicast:
            raise ValueError('a packed output needs `out` and no multicast')
        perm = perm.to(device=device, dtype=torch.int64).contiguous()
        if perm.numel() != n:
            raise ValueError('perm must have a slot per row of v')
        if head_map is not None:
            if head_map.dtype != torch.int32 or head_map.device != device or \
                    head_map.numel() != heads:
                raise ValueError('heads must be int32 ids on the device, one '
                                 'per head of v')
        elif out.shape[1] != heads:
            raise ValueError('out must have v\'s heads')
    if index.shape[0] != heads or count.shape[0] != heads:
        raise ValueError(f'lists for {index.shape[0]} heads, attention over '
                         f'{heads}')
    if out is None:
        out = torch.empty(n, heads, HEAD_DIM, dtype=v.dtype, device=device)
    _check_rows(out, 'out')
    if out.dtype != v.dtype:
        raise ValueError('out must have v\'s dtype')
    index = index.to(torch.int32).contiguous()
    count = count.to(torch.int32).contiguous()
    valid = valid_count.to(torch.int32).contiguous()
    head = (_ptr(q_i8), _ptr(q_scale), _ptr(k_i8), _ptr(k_scale), _ptr(v),
            _DTYPES[v.dtype], v.stride(0), v.stride(1), _ptr(index),
            index.shape[-1], _ptr(count), _ptr(valid), heads, n_tiles,
            _ptr(out))
    tail = (out.stride(0), out.stride(1), _ptr(status_word(device)),
            _stream(device))
    if out_multicast:
        _call(device, 'veda_sparse_attention_multicast', *head,
              ctypes.c_void_p(out_multicast), *tail)
    elif perm is not None:
        _call(device, 'veda_sparse_attention_packed', *head, out.stride(0),
              out.stride(1), _ptr(perm), out.shape[0], _ptr(head_map),
              *tail[2:])
    else:
        _call(device, 'veda_sparse_attention', *head, *tail)
    return out


def gather_tiles(x: torch.Tensor, perm: torch.Tensor,
                 heads: torch.Tensor) -> torch.Tensor:
    """[S, H, 128] -> [N, H', 128] tile order, padding slots zero."""
    _check_rows(x, 'x')
    device = require_device(x, perm, heads)
    perm = perm.to(torch.int64).contiguous()
    heads = heads.to(torch.int64).contiguous()
    out = torch.empty(perm.numel(), heads.numel(), HEAD_DIM, dtype=x.dtype,
                      device=device)
    _call(device, 'veda_gather_tiles', _ptr(x), _DTYPES[x.dtype], x.stride(0),
              x.stride(1), x.shape[0], x.shape[1], _ptr(perm), perm.numel(),
              _ptr(heads), heads.numel(), _ptr(out), _stream(device))
    return out


def scatter_tiles_(out: torch.Tensor, tiled: torch.Tensor, perm: torch.Tensor,
                   heads: torch.Tensor) -> None:
    """out[perm[slot], heads[j]] = tiled[slot, j] for the real slots."""
    _check_rows(out, 'out')
    device = require_device(out, tiled, perm, heads)
    perm = perm.to(torch.int64).contiguous()
    heads = heads.to(torch.int64).contiguous()
    tiled = tiled.contiguous()
    _call(device, 'veda_scatter_tiles', _ptr(tiled), _DTYPES[tiled.dtype],
              _ptr(perm), perm.numel(), _ptr(heads), heads.numel(),
              out.shape[1], _ptr(out), out.stride(0), out.stride(1),
              out.shape[0], _stream(device))
