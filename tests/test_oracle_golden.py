"""The oracle pinned against the fixtures made from the reference's own code
(tests/golden/make_golden.py). CPU only.

  * selection: the oracle's lists equal the reference's on every row whose
    kept set does not depend on the order of equal scores at the k-th place
    (torch.topk leaves that order unspecified); those rows are counted.
  * budgets: split_budget, the ratio budget and the Bresenham pattern equal
    the reference's values exactly.
  * quantisation: int8 codes and scales equal the reference Triton kernel's
    (run under Triton's interpreter) bit for bit.
  * attention: the oracle's INT8 model matches the reference INT8 kernel's
    output within the attention tolerance, and its fp32 masked attention
    matches the reference's fp32 attention to fp16 storage precision.
  * predictor: pooling and logits within fp32 rounding.
"""

import numpy as np
import pytest
import torch

import helpers
import problems
from oracle import attention as oatt
from oracle import int8 as oint8
from oracle import predictor as opred
from oracle import selection as osel


@pytest.fixture(scope='module')
def meta():
    return helpers.meta()


@pytest.mark.parametrize('name', [n for n in problems.CASES
                                  if problems.CASES[n].heads * problems.CASES[
                                      n].seq_len <= 24 * 32768])
def test_selection_matches_reference(meta, name):
    case = problems.CASES[name]
    info = meta['selection'][name]
    scores = problems.make_scores(case)
    assert problems.sha256(scores) == info['scores_sha256'], \
        'score regeneration drifted (torch RNG changed?)'
    layout = case.layout()
    blocks = case.blocks(layout)
    index, count = osel.index_lists(scores, layout, blocks)
    got = helpers.lists_to_mask(index, count, layout.n_tiles)
    want = helpers.golden_mask(helpers.golden('selection'), name,
                               layout.n_tiles)
    ties = np.zeros(count.shape, dtype=bool)
    ties[:, :layout.n_video_tiles] = osel.boundary_ties(scores, layout,
                                                        blocks)
    same = (got == want).all(-1)
    assert same[~ties].all()
    assert int(ties.sum()) == info['boundary_tie_rows']
    assert np.array_equal(
        count, helpers.golden('selection')[f'{name}.count'].astype(np.int32))
    assert int(count.max()) <= osel.max_width(layout, blocks)


def test_selection_large_case_matches_reference(meta):
    name = 'cfg3_131k'
    case = problems.CASES[name]
    scores = problems.make_scores(case)
    assert problems.sha256(scores) == meta['selection'][name]['scores_sha256']
    layout = case.layout()
    index, count = osel.index_lists(scores, layout, case.blocks(layout))
    got = helpers.lists_to_mask(index, count, layout.n_tiles)
    want = helpers.golden_mask(helpers.golden('selection'), name,
                               layout.n_tiles)
    assert np.array_equal(got, want)


def test_tie_rows_are_where_torch_topk_order_decides(meta):
    info = meta['selection']['ties']
    assert info['boundary_tie_rows'] > 0
    assert info['oracle_rows_differing_outside_ties'] == 0


def test_budget_rules_match_reference(meta):
    table = meta['budgets']
    for budget, n_cols, want in table['split_budget']:
        assert list(osel.split_budget(budget, n_cols)) == want
    for ratio, real, n_cols, want in table['per_row']:
        assert osel.Budget(ratio=ratio).per_row(real, n_cols) == want
    for key, bits in table['bresenham_packbits'].items():
        n_rows, frac = key.split(':')
        got = osel.bresenham_extra(int(n_rows), float(frac))
        assert np.array_equal(np.packbits(got), np.array(bits, np.uint8))


def test_reference_unit_pins():
    """The reference's own assertions (tests/unit/test_core_selection.py)."""
    assert osel.split_budget(2.3, 10) == (2, 3, 0.3)
    assert osel.split_budget(12, 10) == (10, 10, 0.0)
    assert osel.split_budget(0.2, 10)[0] == 1
    assert int(osel.bresenham_extra(1000, 0.3).sum()) == 300
    assert osel.Budget(ratio=0.1).per_row(320, 4) == pytest.approx(0.225)


def test_quantize_matches_reference_kernel_bit_exact(meta):
    gold = helpers.golden('quant')
    x = problems.quant_input()
    assert problems.sha256(x) == meta['quant']['input_sha256']
    xf = x.float().numpy()
    qi, qs = oint8.quantize(xf, 128, meta['quant']['pre_scale'])
    ki, ks = oint8.quantize(xf, 64)
    assert np.array_equal(qi, gold['q_int8'])
    assert np.array_equal(qs, gold['q_scale'])
    assert np.array_equal(ki, gold['k_int8'])
    assert np.array_equal(ks, gold['k_scale'])
    # the planted zero block gets scale 1 and zero codes
    assert (qs[1, 1] == 1.0) and (qi[128:256, 1] == 0).all()


@pytest.mark.parametrize('name', ['selftest', 'cfg0', 'gpu_problem'])
def test_attention_models_match_reference(meta, name):
    case = problems.CASES[name]
    q, k, v, scores, layout = problems.make_problem(case)
    assert problems.sha256(q, k, v) == meta['attention'][name]['qkv_sha256']
    index, count = osel.index_lists(scores, layout, case.blocks(layout))
    gold = helpers.golden('attention')
    rows = gold[f'{name}.rows']
    real = layout.slot_valid[rows]
    qf, kf, vf = (t.float().numpy() for t in (q, k, v))
    # gpu_problem is checked on its first head to keep the CPU suite short
    heads = None if name != 'gpu_problem' else [0]
    cols = slice(None) if heads is None else slice(0, 1)
    model = oint8.int8_block_sparse(qf, kf, vf, index, count,
                                    layout.valid_count, heads=heads)
    m = helpers.compare(model[rows][real][:, cols],
                        gold[f'{name}.int8_out'].astype(np.float32)[real]
                        [:, cols])
    within = helpers.within_selftest_tolerance if name == 'selftest' else \
        helpers.within_int8_tolerance
    assert within(m), m
    mask = oatt.mask_from_lists(index, count, layout.n_tiles)
    exact = oatt.block_sparse_attention(qf, kf, vf, mask, layout.slot_valid,
                                        heads=heads)
    want = gold[f'{name}.fp32_out'].astype(np.float32)[real][:, cols]
    got = exact[rows][real][:, cols]
    np.testing.assert_allclose(got, want, atol=4e-3, rtol=2e-3)


@pytest.mark.parametrize('name', ['selftest', 'gpu_problem'])
def test_predictor_matches_reference(name):
    case = problems.CASES[name]
    q, k, _, _, layout = problems.make_problem(case)
    gold = helpers.golden('predictor')
    fq = opred.pool_video_tiles(q.float().numpy(), layout)
    fk = opred.pool_video_tiles(k.float().numpy(), layout)
    np.testing.assert_allclose(fq, gold[f'{name}.feats_q'], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(fk, gold[f'{name}.feats_k'], rtol=1e-5,
                               atol=1e-6)
    proj = problems.make_proj(case).float().numpy()
    logits = opred.tile_logits(gold[f'{name}.feats_q'],
                               gold[f'{name}.feats_k'], proj[0], proj[1])
    np.testing.assert_allclose(logits, gold[f'{name}.logits'], rtol=1e-4,
                               atol=1e-5)


def test_problems_regenerate_identically():
    a = problems.make_scores(problems.CASES['cfg0'])
    b = problems.make_scores(problems.CASES['cfg0'])
    assert np.array_equal(a, b)
    assert torch.equal(problems.quant_input(), problems.quant_input())
