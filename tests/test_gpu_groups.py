"""A layer whose heads use two tile shapes (a tile plan's head groups,
core/plans.py:25-29), through one `VedaAttention.attention` call.

The result must equal, bit for bit, per-group `layer` calls on copies of
each group's heads scattered back; the call copies nothing (the head ids go
to the kernels). Its selection statistics must equal the reference's own
`Stats` (core/engine.py:48-107) fed by the reference's own selection on the
same scores, when the reference package is in baseline/_ref.
"""

import os
import sys

import pytest
import torch

import conftest

pytestmark = pytest.mark.gpu

REF = os.path.join(conftest.REPO, 'baseline', '_ref')
SEQ = 300 + 4 * 16 * 24
SPANS = [(300, (4, 16, 24))]          # text 300 rows (global), target 4x16x24
SHAPES = [(1, 8, 16), (2, 8, 8)]
GROUPS = [[0, 2, 5], [1, 3, 4]]


def _layouts(device):
    from veda_b200 import tiling
    return [tiling.build_tile_layout(
        [tiling.TiledSpan(s, g, tiling.TileShape(*shape)) for s, g in SPANS],
        SEQ, device) for shape in SHAPES]


def _inputs(device, layouts, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(31)
    q, k, v = (torch.randn(SEQ, 6, 128, generator=g).to(dtype)
               .to(device) for _ in range(3))
    scores = [torch.rand(3, lay.n_video_tiles, lay.n_video_tiles,
                         generator=g).to(device) for lay in layouts]
    return q, k, v, scores


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
def test_two_shape_layer_equals_per_group_calls(cuda_device, dtype):
    from veda_b200 import engine, ops, selection
    layouts = _layouts(cuda_device)
    q, k, v, scores = _inputs(cuda_device, layouts, dtype)
    budget = selection.Budget(ratio=0.3)
    attn = engine.VedaAttention(budget)
    groups = [engine.HeadGroup(lay, heads, scores=s)
              for lay, heads, s in zip(layouts, GROUPS, scores)]
    got = attn.attention(q, k, v, groups)
    again = attn.attention(q, k, v, groups)
    want = torch.empty_like(got)
    single = engine.VedaAttention(budget)
    for lay, heads, s in zip(layouts, GROUPS, scores):
        idx = torch.tensor(heads, device=cuda_device)
        want[:, idx] = single.layer(q[:, idx].contiguous(),
                                    k[:, idx].contiguous(),
                                    v[:, idx].contiguous(), lay, scores=s,
                                    tiled=False)
    ops.check_status(cuda_device)
    assert torch.equal(got, want)
    assert torch.equal(got, again)


def test_two_shape_full_layer_equals_per_group_calls(cuda_device):
    from veda_b200 import engine, selection
    layouts = _layouts(cuda_device)
    q, k, v, _ = _inputs(cuda_device, layouts)
    attn = engine.VedaAttention(selection.Budget(ratio=0.3))
    got = attn.attention(q, k, v, [engine.HeadGroup(lay, heads)
                                   for lay, heads in zip(layouts, GROUPS)],
                         full=True)
    want = torch.empty_like(got)
    for lay, heads in zip(layouts, GROUPS):
        idx = torch.tensor(heads, device=cuda_device)
        want[:, idx] = attn.layer(q[:, idx].contiguous(),
                                  k[:, idx].contiguous(),
                                  v[:, idx].contiguous(), lay, full=True,
                                  tiled=False)
    assert torch.equal(got, want)


def test_stats_equal_the_reference_stats(cuda_device):
    if not os.path.isdir(os.path.join(REF, 'veda_comfy')):
        pytest.skip('the reference package is not in baseline/_ref')
    if REF not in sys.path:
        sys.path.append(REF)
    try:
        from veda_comfy.core import engine as rengine
        from veda_comfy.core import selection as rsel
        from veda_comfy.core import tiling as rtil
    except ImportError as e:
        pytest.skip(f'the reference package does not import: {e}')
    from veda_b200 import engine, selection
    layouts = _layouts(cuda_device)
    q, k, v, scores = _inputs(cuda_device, layouts)
    attn = engine.VedaAttention(selection.Budget(ratio=0.3))
    attn.attention(q, k, v, [engine.HeadGroup(lay, heads, scores=s)
                             for lay, heads, s in zip(layouts, GROUPS,
                                                      scores)])
    ref = rengine.Stats()
    for shape, s in zip(SHAPES, scores):
        rlay = rtil.build_tile_layout(
            [rtil.TiledSpan(st, g, rtil.TileShape(*shape)) for st, g in SPANS],
            SEQ, cuda_device)
        blocks = rsel.column_blocks(rlay, rsel.Budget(ratio=0.3),
                                    rsel.Budget(ratio=1.0))
        _, keep = rsel.select(s, rlay, blocks)
        ref.add(keep, rlay)
    assert attn.stats.per_row() == ref.per_row()
    assert int(attn.stats.kept) == int(ref.kept)
    assert attn.stats.video_pairs == ref.video_pairs
    assert attn.stats.kept_fraction() == ref.kept_fraction()
    assert attn.stats.compute_fraction() == pytest.approx(
        ref.compute_fraction(), rel=1e-12)
