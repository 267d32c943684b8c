"""The packed-row paths against the separate passes they fold in, on a
layout whose permutation is not the identity (spans, padding slots):
quantisation reading packed rows through the permutation, with V copied
into tile order by the same launch, equals gather_tiles then quantisation;
the attention epilogue writing through the permutation equals the
attention then scatter_tiles_; bit for bit."""

import pytest
import torch

import helpers
import problems

pytestmark = pytest.mark.gpu


def _packed(case, dtype, device):
    gen = torch.Generator().manual_seed(case.seed)
    return tuple(t.to(dtype).to(device) for t in problems.packed_qkv(case, gen))


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
def test_packed_quantisation_equals_gather_then_quantisation(cuda_device,
                                                              dtype):
    from veda_b200 import kernels, ops
    case = problems.CASES['gpu_problem']
    layout = helpers.device_layout(case, cuda_device)
    assert not layout.identity
    q, k, v = _packed(case, dtype, cuda_device)
    heads = torch.arange(q.shape[1], device=cuda_device)
    pre = 128 ** -0.5 * kernels.LOG2E
    want = ops.quant_pool(ops.gather_tiles(q, layout.perm, heads),
                          ops.gather_tiles(k, layout.perm, heads),
                          layout.valid_count, layout.n_video_tiles, pre)
    got = ops.quant_pool(q, k, layout.valid_count, layout.n_video_tiles, pre,
                         perm=layout.perm, v=v)
    for key in ('q_i8', 'q_scale', 'k_i8', 'k_scale', 'feats_q', 'feats_k'):
        assert torch.equal(got[key], want[key]), key
    assert torch.equal(got['v_tiled'], ops.gather_tiles(v, layout.perm,
                                                        heads))


@pytest.mark.parametrize('view', ['fused_qkv', 'head_major'])
def test_packed_v_copy_of_a_head_group_on_strided_v(cuda_device, view):
    """A head group's V copied into tile order from V viewed out of a fused
    [S, 3H, 128] projection or out of a head-major [H, S, 128] buffer,
    against gather_tiles of the same heads."""
    from veda_b200 import ops
    case = problems.CASES['gpu_problem']
    layout = helpers.device_layout(case, cuda_device)
    q, k, v = _packed(case, torch.bfloat16, cuda_device)
    n_heads = v.shape[1]
    group = [n_heads - 1, 0] if n_heads > 1 else [0]
    ids32 = ops.head_ids(group, n_heads, cuda_device)
    if view == 'fused_qkv':
        v_view = torch.cat([q, k, v], dim=1)[:, 2 * n_heads:]
    else:
        v_view = v.transpose(0, 1).contiguous().transpose(0, 1)
    assert torch.equal(v_view, v) and not v_view.is_contiguous()
    got = ops.quant_pool(q, k, layout.valid_count, 0, 0.1, pool=False,
                         perm=layout.perm, heads=ids32, v=v_view)
    ops.check_status(cuda_device)
    assert torch.equal(got['v_tiled'],
                       ops.gather_tiles(v, layout.perm, ids32.to(torch.int64)))


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
def test_packed_output_equals_attention_then_scatter(cuda_device, dtype):
    from veda_b200 import kernels, ops
    from veda_b200 import selection as vs
    case = problems.CASES['gpu_problem']
    layout = helpers.device_layout(case, cuda_device)
    q, k, v, scores, _ = problems.make_problem(case)
    q, k, v = (t.to(dtype).to(cuda_device) for t in (q, k, v))
    index, count = vs.select_index(torch.from_numpy(scores).to(cuda_device),
                                   layout, helpers.product_blocks(case, layout))
    quant = ops.quant_pool(q, k, layout.valid_count, 0,
                           128 ** -0.5 * kernels.LOG2E, pool=False)
    args = (quant['q_i8'], quant['q_scale'], quant['k_i8'], quant['k_scale'],
            v, index, count, layout.valid_count)
    tiled = ops.sparse_attention(*args)
    heads = torch.arange(v.shape[1], device=cuda_device)
    want = torch.zeros(case.seq_len, v.shape[1], 128, dtype=dtype,
                       device=cuda_device)
    ops.scatter_tiles_(want, tiled, layout.perm, heads)
    got = torch.zeros_like(want)
    ops.sparse_attention(*args, out=got, perm=layout.perm)
    ops.check_status(cuda_device)
    assert torch.equal(got, want)


@pytest.mark.parametrize('pool', [False, True])
def test_packed_quantisation_of_an_odd_head_group(cuda_device, pool):
    """Three heads of four, in a scrambled order: the two-heads-per-CTA
    launch leaves its last CTA's second head out. Codes, scales, features
    and the V copy equal gather_tiles then quantisation of the same heads."""
    from veda_b200 import kernels, ops
    case = problems.CASES['gpu_problem']
    layout = helpers.device_layout(case, cuda_device)
    q, k, v = _packed(case, torch.bfloat16, cuda_device)
    n_heads = q.shape[1]
    group = [2, 0, 3][:max(1, n_heads - 1)]
    ids32 = ops.head_ids(group, n_heads, cuda_device)
    ids64 = ids32.to(torch.int64)
    pre = 128 ** -0.5 * kernels.LOG2E
    n_video = layout.n_video_tiles if pool else 0
    want = ops.quant_pool(ops.gather_tiles(q, layout.perm, ids64),
                          ops.gather_tiles(k, layout.perm, ids64),
                          layout.valid_count, n_video, pre, pool=pool)
    got = ops.quant_pool(q, k, layout.valid_count, n_video, pre, pool=pool,
                         perm=layout.perm, heads=ids32, v=v)
    ops.check_status(cuda_device)
    keys = ['q_i8', 'q_scale', 'k_i8', 'k_scale'] + \
        (['feats_q', 'feats_k'] if pool else [])
    for key in keys:
        assert torch.equal(got[key], want[key]), key
    assert torch.equal(got['v_tiled'], ops.gather_tiles(v, layout.perm, ids64))
