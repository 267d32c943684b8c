"""Host-side logic of the product (`veda_b200`), on CPU.

  * budgets, Bresenham rows and column blocks equal the reference's values
    (fixtures made from the reference's own code) and the oracle's;
  * tile layouts equal the oracle's for every test geometry, and a layout
    converted from the reference's own fields is the same layout;
  * index-list widths fit every row the reference keeps;
  * the kernel package helpers (`key_blocks`, `dense_index`,
    `mask_from_lists`) give the reference's expansions;
  * the error behaviour of the boundary without a GPU: `create()` raises
    BackendUnavailable, a missing library raises LibraryMissing (a
    MissingDependency at `create()`), CPU tensors are refused.
"""

import types

import numpy as np
import pytest
import torch

import helpers
import problems
from oracle import selection as osel


def _product_budget(b):
    from veda_b200 import selection as vs
    return vs.Budget(ratio=b.ratio) if b.tiles is None else vs.Budget(
        tiles=b.tiles)


def test_budget_rules_equal_the_reference():
    from veda_b200 import selection as vs
    table = helpers.meta()['budgets']
    for budget, n_cols, want in table['split_budget']:
        assert list(vs.split_budget(budget, n_cols)) == want
    for ratio, real, n_cols, want in table['per_row']:
        assert vs.Budget(ratio=ratio).per_row(real, n_cols) == want
    for key, bits in table['bresenham_packbits'].items():
        n_rows, frac = key.split(':')
        got = vs.bresenham_extra(int(n_rows), float(frac), 'cpu').numpy()
        assert np.array_equal(np.packbits(got.astype(bool)),
                              np.array(bits, np.uint8))


def test_reference_unit_pins_hold_for_the_product():
    """tests/unit/test_core_selection.py:24-97 of the reference."""
    from veda_b200 import selection as vs
    assert vs.split_budget(2.3, 10) == (2, 3, 0.3)
    assert vs.split_budget(12, 10) == (10, 10, 0.0)
    assert vs.split_budget(0.2, 10)[0] == 1
    assert int(vs.bresenham_extra(1000, 0.3, 'cpu').sum()) == 300
    assert vs.Budget(ratio=0.1).per_row(320, 4) == pytest.approx(0.225)
    assert vs.Budget.sparsity(90).ratio == pytest.approx(0.1)
    with pytest.raises(ValueError):
        vs.Budget()
    with pytest.raises(ValueError):
        vs.Budget(ratio=0.5, tiles=3)
    with pytest.raises(ValueError):
        vs.Budget.sparsity(100)


@pytest.mark.parametrize('name', list(problems.CASES))
def test_layout_equals_oracle(name):
    case = problems.CASES[name]
    want = case.layout()
    got = helpers.device_layout(case, 'cpu')
    assert np.array_equal(got.perm.numpy(), want.perm)
    assert np.array_equal(got.valid_count.numpy(), want.valid_count)
    assert (got.n_video_tiles, got.n_ref_tiles, got.n_global_tiles) == (
        want.n_video_tiles, want.n_ref_tiles, want.n_global_tiles)
    assert (got.ref_tokens, got.target_tokens, got.seq_len) == (
        want.ref_tokens, want.target_tokens, want.seq_len)
    assert np.array_equal(got.kv_ok.numpy(), want.kv_ok)
    assert np.array_equal(got.slot_valid.numpy(), want.slot_valid)
    assert got.num_slots == want.num_slots


def test_layout_from_reference_fields():
    from veda_b200 import tiling as vt
    case = problems.CASES['gpu_problem']
    ours = helpers.device_layout(case, 'cpu')
    # the reference's TileLayout carries these fields (core/tiling.py:115-168)
    ref = types.SimpleNamespace(
        perm=ours.perm.clone(), valid_count=ours.valid_count.clone(),
        n_video_tiles=ours.n_video_tiles, n_ref_tiles=ours.n_ref_tiles,
        n_global_tiles=ours.n_global_tiles, ref_tokens=ours.ref_tokens,
        target_tokens=ours.target_tokens, seq_len=ours.seq_len,
        gather_index=ours.perm.clamp(min=0))
    got = vt.from_reference(ref)
    assert torch.equal(got.perm, ours.perm)
    assert torch.equal(got.valid_count, ours.valid_count)
    assert torch.equal(got.kv_ok, ours.kv_ok)
    assert got.identity == ours.identity


def test_layout_rejects_overlapping_spans():
    from veda_b200 import tiling as vt
    spans = [vt.TiledSpan(0, (1, 8, 16), vt.TileShape(1, 8, 16)),
             vt.TiledSpan(64, (1, 8, 16), vt.TileShape(1, 8, 16))]
    with pytest.raises(ValueError):
        vt.build_tile_layout(spans, 400)
    with pytest.raises(ValueError):
        vt.build_tile_layout([], 400)


@pytest.mark.parametrize('name', list(problems.CASES))
def test_blocks_and_width_fit_the_reference(name):
    """Column blocks match the oracle's, the kernel's (k_lo, Bresenham) rows
    give the reference's per-row counts, and the list width holds every
    row the reference keeps."""
    from veda_b200 import selection as vs
    case = problems.CASES[name]
    olayout = case.layout()
    layout = helpers.device_layout(case, 'cpu')
    oblocks = case.blocks(olayout)
    blocks = helpers.product_blocks(case, layout)
    assert [(b.start, b.stop, b.real_tokens) for b in blocks] == [
        (b.start, b.stop, b.real_tokens) for b in oblocks]
    spec, extra = vs.kernel_blocks(layout, blocks, 'cpu')
    for (start, stop, keeps_all, k_lo), b, row in zip(spec, oblocks, extra):
        n_cols = stop - start
        if keeps_all:
            assert b.budget.keeps_all and k_lo == n_cols
            continue
        lo, _, frac = osel.split_budget(
            b.budget.per_row(b.real_tokens, n_cols), n_cols)
        assert k_lo == lo
        assert np.array_equal(row.numpy().astype(bool),
                              osel.bresenham_extra(olayout.n_video_tiles,
                                                   frac))
    width = vs.list_width(layout, blocks)
    count = helpers.golden('selection')[f'{name}.count']
    assert int(count.max()) <= width <= layout.n_tiles
    assert width == osel.max_width(olayout, oblocks)


def test_key_blocks_expand_tiles_to_64_row_blocks():
    """kernels.key_blocks is the reference's host expansion
    (sparse_int8.py:295-309): tile t -> blocks 2t, 2t+1, their valid rows."""
    from veda_b200 import kernels
    index = torch.tensor([[[0, 2, -1], [1, 2, 3]]], dtype=torch.int32)
    count = torch.tensor([[2, 3]], dtype=torch.int32)
    valid = torch.tensor([128, 128, 100, 0], dtype=torch.int32)
    blocks, bcount, bvalid = kernels.key_blocks(index, count, valid)
    assert blocks[0, 0, :4].tolist() == [0, 1, 4, 5]
    assert blocks[0, 1].tolist() == [2, 3, 4, 5, 6, 7]
    assert bcount.tolist() == [[4, 6]]
    assert bvalid.tolist() == [64, 64, 64, 64, 64, 36, 0, 0]


def test_dense_index_keeps_every_non_empty_tile():
    from veda_b200 import selection as vs
    case = problems.CASES['cfg4']
    layout = helpers.device_layout(case, 'cpu')
    index, count = vs.dense_index(layout, 3)
    kv = np.flatnonzero(layout.kv_ok.numpy())
    assert index.shape == (3, layout.n_tiles, kv.size)
    assert (count == kv.size).all()
    assert np.array_equal(index[2, 5].numpy(), kv)


def test_mask_from_lists_round_trip():
    from veda_b200 import backend
    g = torch.Generator().manual_seed(4)
    mask = torch.rand(2, 9, 9, generator=g) < 0.3
    count = mask.sum(-1).to(torch.int32)
    width = int(count.max())
    index = torch.full((2, 9, width), -1, dtype=torch.int32)
    for h in range(2):
        for r in range(9):
            ids = torch.nonzero(mask[h, r]).view(-1)
            index[h, r, :ids.numel()] = ids.to(torch.int32)
    assert torch.equal(backend.mask_from_lists(index, count, 9), mask)


def test_reference_attention_helper_matches_oracle():
    """backend.reference_attention (the self-test's yardstick) equals the
    oracle's fp32 masked attention (core/reference.py:14-36)."""
    from oracle import attention as oatt
    from veda_b200 import backend
    case = problems.CASES['selftest']
    layout = helpers.device_layout(case, 'cpu')
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(layout.num_slots, 2, 128, generator=g)
               * layout.slot_valid[:, None, None] for _ in range(3))
    mask = torch.rand(2, layout.n_tiles, layout.n_tiles, generator=g) < 0.4
    got = backend.reference_attention(q, k, v, mask, layout).numpy()
    sv = layout.slot_valid.numpy().astype(bool)
    for h in range(q.shape[1]):
        want = oatt.block_sparse_head(q[:, h].numpy(), k[:, h].numpy(),
                                      v[:, h].numpy(), mask[h].numpy(), sv)
        np.testing.assert_allclose(got[:, h], want, rtol=1e-4, atol=1e-5)


def test_create_without_a_gpu_is_backend_unavailable():
    from veda_b200 import backend
    if torch.cuda.is_available():
        pytest.skip('a GPU is present')
    with pytest.raises(backend.BackendUnavailable):
        backend.create()


def test_missing_library_is_a_missing_dependency(monkeypatch, tmp_path):
    from veda_b200 import _lib, backend
    monkeypatch.setattr(_lib, 'LIBRARY', str(tmp_path / 'absent.so'))
    monkeypatch.setattr(_lib, '_lib', None)
    with pytest.raises(_lib.LibraryMissing):
        _lib.load()
    if torch.cuda.is_available():
        with pytest.raises(backend.MissingDependency):
            backend.create()


def test_ops_refuse_cpu_tensors():
    from veda_b200 import ops
    x = torch.zeros(128, 1, 128, dtype=torch.bfloat16)
    with pytest.raises((ValueError, RuntimeError)):
        ops.quantize(x, 128)
