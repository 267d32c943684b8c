"""Whole-path parity on the GPU at the benchmark's full sizes, through the
product API (engine, backend, kernel package) and so through the C ABI.

The oracle cannot evaluate a 32k-token layer in a test's time, so at full
size the checks are properties that hold at any size:
  * index lists of every row equal the oracle's (bit-exact);
  * int8 codes and scales of sampled tiles equal the oracle's (bit-exact);
  * attention of sampled (head, query tile) pairs is within the attention
    tolerance of the oracle's INT8 model on the same lists;
  * repeated calls give identical bits; full density equals the dense walk;
  * the packed-input path (gather, attend, scatter) equals the tile-order
    path bit for bit.
Cases: cfg1 (config 1), the full-attention layer of config 2 at cfg1 size,
config 3 at 131,072 tokens, config 4 (generated + global reference tiles),
and the self-test problem through `Backend.attend`.
"""

import numpy as np
import pytest
import torch

import helpers
import problems
from oracle import attention as oatt
from oracle import int8 as oint8
from oracle import selection as osel
from oracle import tiling as otil

pytestmark = pytest.mark.gpu


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _case_on_device(name, device):
    case = problems.CASES[name]
    q, k, v, scores, olayout = problems.make_problem(case)
    layout = helpers.device_layout(case, device)
    return case, (q, k, v), scores, olayout, layout


def _engine(case):
    from veda_b200 import engine
    blocks = helpers.product_blocks(case, helpers.device_layout(case, 'cpu'))
    gen = blocks[-1].budget
    ref = blocks[0].budget if len(blocks) > 1 else None
    return engine.VedaAttention(gen, ref) if ref else engine.VedaAttention(
        gen)


def _check_sampled(out, qkv, index, count, valid, heads, q_tiles,
                   slot_valid):
    q, k, v = (t.float().numpy() for t in qkv)
    want = oint8.int8_block_sparse(q, k, v, index, count, valid,
                                   heads=heads, q_tiles=q_tiles)
    rows = np.concatenate([np.arange(t * 128, (t + 1) * 128)
                           for t in q_tiles])
    rows = rows[slot_valid[rows]]
    for h in heads:
        m = helpers.compare(out[rows, h], want[rows, h])
        assert helpers.within_int8_tolerance(m), (h, m)


def test_cfg1_call_matches_oracle(cuda_device):
    """Config 1 end to end: 24 heads, 32,760 tokens, 26 of 256 tiles."""
    from veda_b200 import kernels
    case, qkv, scores, olayout, layout = _case_on_device('cfg1', cuda_device)
    attn = _engine(case)
    dq, dk, dv = (t.to(cuda_device) for t in qkv)
    dscores = torch.from_numpy(scores).to(cuda_device)
    out = attn.layer(dq, dk, dv, layout, scores=dscores)
    again = attn.layer(dq, dk, dv, layout, scores=dscores)
    assert torch.equal(out, again)                   # deterministic
    index, count = attn.select(dscores, layout)
    index, count = index.cpu().numpy(), count.cpu().numpy()
    oidx, ocnt = osel.index_lists(scores, olayout, case.blocks(olayout))
    assert np.array_equal(count, ocnt)
    assert np.array_equal(helpers.lists_to_mask(index, count, 256),
                          helpers.lists_to_mask(oidx, ocnt, 256))
    # every int8 code and scale of Q (128-row blocks) and K (64-row blocks)
    for x, block, pre in [(0, 128, oint8.q_pre_scale(128)), (1, 64, 1.0)]:
        qi, qs = kernels.quantize(dq if x == 0 else dk, block, float(pre))
        oqi, oqs = oint8.quantize(qkv[x].float().numpy(), block, pre)
        assert np.array_equal(qi.cpu().numpy(), oqi.transpose(1, 0, 2))
        assert np.array_equal(qs.cpu().numpy(), oqs)
    _check_sampled(_np(out), qkv, index, count, olayout.valid_count,
                   [0, 11, 23], [0, 97, 255], olayout.slot_valid.astype(bool))


def test_full_attention_layer_at_cfg1_size(cuda_device):
    """A full_attention_layers layer (config 2's layers 0, 1, 47): every
    non-empty key tile, through the same kernel."""
    case, qkv, scores, olayout, layout = _case_on_device('cfg1', cuda_device)
    attn = _engine(case)
    qkv6 = tuple(t[:, :6].contiguous() for t in qkv)
    dq, dk, dv = (t.to(cuda_device) for t in qkv6)
    out = attn.layer(dq, dk, dv, layout, full=True)
    index = np.tile(np.arange(256, dtype=np.int32), (6, 256, 1))
    count = np.full((6, 256), 256, dtype=np.int32)
    _check_sampled(_np(out), qkv6, index, count, olayout.valid_count,
                   [0, 5], [1, 255], olayout.slot_valid.astype(bool))


def test_dense_walk_matches_fp32_attention(cuda_device):
    """Config 0's shape at 100% density against fp32 dense attention, with
    the reference backend's bound (5% of absmax)."""
    case, qkv, scores, olayout, layout = _case_on_device('cfg0', cuda_device)
    attn = _engine(case)
    out = _np(attn.layer(*(t.to(cuda_device) for t in qkv), layout,
                         full=True))
    mask = np.ones((4, 32, 32), dtype=bool)
    want = oatt.block_sparse_attention(*(t.float().numpy() for t in qkv),
                                       mask, olayout.slot_valid.astype(bool))
    m = helpers.compare(out, want)
    assert m['max_rel'] < 0.05 and m['cos'] > 0.999, m


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
def test_long_clip_131k(cuda_device, dtype):
    """Config 3 at 131,072 tokens: 1,024 tiles, 90% sparse (102.4 per row:
    102 or 103 by the Bresenham pattern)."""
    case, qkv, scores, olayout, layout = _case_on_device('cfg3_131k',
                                                         cuda_device)
    qkv = tuple(t.to(dtype) for t in qkv)
    attn = _engine(case)
    dscores = torch.from_numpy(scores).to(cuda_device)
    out = attn.layer(*(t.to(cuda_device) for t in qkv), layout,
                     scores=dscores)
    index, count = attn.select(dscores, layout)
    index, count = index.cpu().numpy(), count.cpu().numpy()
    assert set(np.unique(count)) == {102, 103}
    _check_sampled(_np(out), qkv, index, count, olayout.valid_count,
                   [0, 1], [0, 600, 1023], olayout.slot_valid.astype(bool))


def test_cfg4_generated_plus_global_reference_tiles(cuda_device):
    """Config 4: 192 generated tiles (top 32) + 64 global reference tiles
    (reference_sparsity 0%): generated rows walk 32 + 64 tiles, global rows
    walk all 256."""
    case, qkv, scores, olayout, layout = _case_on_device('cfg4', cuda_device)
    attn = _engine(case)
    dscores = torch.from_numpy(scores).to(cuda_device)
    # N == S here, so the tile order is stated rather than inferred
    out = attn.layer(*(t.to(cuda_device) for t in qkv), layout,
                     scores=dscores, tiled=True)
    index, count = attn.select(dscores, layout)
    index, count = index.cpu().numpy(), count.cpu().numpy()
    assert (count[:, :192] == 96).all() and (count[:, 192:] == 256).all()
    oidx, ocnt = osel.index_lists(scores, olayout, case.blocks(olayout))
    assert np.array_equal(helpers.lists_to_mask(index, count, 256),
                          helpers.lists_to_mask(oidx, ocnt, 256))
    _check_sampled(_np(out), qkv, index, count, olayout.valid_count,
                   [0, 13], [7, 191, 192, 255],
                   olayout.slot_valid.astype(bool))


def test_packed_input_path_equals_tile_order_path(cuda_device):
    """gather -> attend -> scatter on packed [S, H, D] rows gives, row for
    row, the tile-order result (gather / scatter are exact copies)."""
    case = problems.CASES['gpu_problem']
    olayout = case.layout()
    layout = helpers.device_layout(case, cuda_device)
    gen = torch.Generator().manual_seed(case.seed)
    packed = tuple(t.to(cuda_device) for t in problems.packed_qkv(case, gen))
    scores = torch.from_numpy(problems.make_scores(case)).to(cuda_device)
    attn = _engine(case)
    out_packed = attn.layer(*packed, layout, scores=scores)
    tiled = tuple(torch.from_numpy(otil.gather_tiles(
        t.float().cpu().numpy(), olayout)).to(torch.bfloat16).to(cuda_device)
        for t in packed)
    out_tiled = attn.layer(*tiled, layout, scores=scores, tiled=True)
    want = otil.scatter_tiles(_np(out_tiled), olayout)
    assert out_packed.shape[0] >= case.seq_len
    assert np.array_equal(_np(out_packed)[:case.seq_len], want[:case.seq_len])


def test_engine_predictor_path_selects_on_its_own_logits(cuda_device):
    """proj_q / proj_k in: pool -> logits -> select -> attend, and the lists
    equal the oracle's selection on the same logits."""
    from veda_b200 import kernels, ops
    case, qkv, _, olayout, layout = _case_on_device('gpu_problem',
                                                    cuda_device)
    attn = _engine(case)
    proj = problems.make_proj(case).to(cuda_device)
    dq, dk, dv = (t.to(cuda_device) for t in qkv)
    out = attn.layer(dq, dk, dv, layout, proj_q=proj[0], proj_k=proj[1])
    quant = ops.quant_pool(dq, dk, layout.valid_count, layout.n_video_tiles,
                           128 ** -0.5 * kernels.LOG2E, pool=True)
    logits = ops.tile_logits(quant['feats_q'], quant['feats_k'], proj[0],
                             proj[1])
    index, count = attn.select(logits, layout)
    oidx, ocnt = osel.index_lists(logits.cpu().numpy(), olayout,
                                  case.blocks(olayout))
    assert np.array_equal(
        helpers.lists_to_mask(index.cpu().numpy(), count.cpu().numpy(),
                              olayout.n_tiles),
        helpers.lists_to_mask(oidx, ocnt, olayout.n_tiles))
    direct = kernels.attend(dq, dk, dv, index, count, layout.valid_count)
    assert torch.equal(out, direct)


def test_backend_attend_with_a_mask_equals_the_list_path(cuda_device):
    """`Backend.attend` with the reference's dense block mask (the self-test
    problem: mixed spans, partial tiles, global rows) gives the same bits as
    the kernel package on the lists the mask stands for; the reference's
    own self-test of this backend is in test_reference_boundary.py."""
    from veda_b200 import backend, kernels, selection
    case = problems.CASES['selftest']
    q, k, v, scores, olayout = problems.make_problem(case)
    layout = helpers.device_layout(case, cuda_device)
    index, count = selection.select_index(
        torch.from_numpy(scores).to(cuda_device), layout,
        helpers.product_blocks(case, layout))
    mask = backend.mask_from_lists(index, count, layout.n_tiles)
    b = backend.create(cuda_device)
    for dtype in b.dtypes:
        dq, dk, dv = (t.to(dtype).to(cuda_device) for t in (q, k, v))
        out = b.attend(dq, dk, dv, mask, layout)
        lists = selection.tile_index_list(mask, layout.kv_ok)
        assert torch.equal(out, kernels.attend(dq, dk, dv, *lists,
                                               layout.valid_count))
