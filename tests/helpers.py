"""Shared helpers of the tests: fixtures on disk, layouts, error metrics."""

from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f'{name}.npz')) as data:
        return {k: data[k] for k in data.files}


def meta() -> dict:
    with open(os.path.join(GOLDEN, 'meta.json')) as f:
        return json.load(f)


def golden_mask(sel: dict, name: str, n_tiles: int) -> np.ndarray:
    bits = sel[f'{name}.mask_bits']
    return np.unpackbits(bits, axis=-1)[..., :n_tiles].astype(bool)


def device_layout(case, device):
    """The product's TileLayout of a test case."""
    from veda_b200 import tiling as vt
    if case.spans is None:
        real = case.seq_len if case.real is None else case.real
        return vt.identity_layout(real, device)
    spans = [vt.TiledSpan(s, tuple(g), vt.TileShape(*t))
             for s, g, t in case.spans]
    return vt.build_tile_layout(spans, case.seq_len, device)


def product_blocks(case, layout):
    from veda_b200 import selection as vs

    def conv(b):
        return vs.Budget(ratio=b.ratio) if b.tiles is None else vs.Budget(
            tiles=b.tiles)
    return vs.column_blocks(layout, conv(case.generated),
                            conv(case.reference))


def lists_to_mask(index: np.ndarray, count: np.ndarray,
                  n_tiles: int) -> np.ndarray:
    heads, n, width = index.shape
    mask = np.zeros((heads, n, n_tiles), dtype=bool)
    live = np.arange(width)[None, None, :] < count[..., None]
    h, r, c = np.nonzero(live)
    mask[h, r, index[h, r, c]] = True
    return mask


def compare(got: np.ndarray, want: np.ndarray) -> dict:
    """cosine similarity, max |diff|, max |want|, max |diff| / max(1,
    max |want|) and relative L2."""
    g = got.astype(np.float64).ravel()
    w = want.astype(np.float64).ravel()
    cos = float(g @ w / max(np.linalg.norm(g) * np.linalg.norm(w), 1e-30))
    diff = np.abs(g - w)
    return {'cos': cos, 'max_abs': float(diff.max()) if diff.size else 0.0,
            'absmax': float(np.abs(w).max()) if w.size else 0.0,
            'max_rel': float(diff.max() / max(np.abs(w).max(), 1.0))
            if diff.size else 0.0,
            'rel_l2': float(np.linalg.norm(g - w) / max(np.linalg.norm(w),
                                                        1e-30))}


COS_MIN = 0.9995
MAX_ABS = 2e-2


def within_int8_tolerance(m: dict) -> bool:
    """The attention tolerance of every benchmark configuration: cos >=
    0.9995 and max |diff| <= 2e-2, flat (not scaled by the output)."""
    return m['cos'] >= COS_MIN and m['max_abs'] <= MAX_ABS


def within_selftest_tolerance(m: dict) -> bool:
    """The same bar scaled by the output's magnitude, for the reference's
    self-test problem only: its inputs are 1.5 N(0,1), and there the
    reference's own Triton kernel and its own INT8 model already differ by
    0.029, because the kernel sums each 64-key block of P V in fp16, an
    error that grows with the output."""
    return m['cos'] >= COS_MIN and m['max_abs'] <= MAX_ABS * max(
        1.0, m['absmax'])
