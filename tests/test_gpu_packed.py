"""The packed-row paths against the separate passes they fold in, on a
layout whose permutation is not the identity (spans, padding slots):
quantisation reading packed rows through the permutation equals
gather_tiles then quantisation, and the attention epilogue writing through
the permutation equals the attention then scatter_tiles_, bit for bit."""

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
    q, k, _ = _packed(case, dtype, cuda_device)
    heads = torch.arange(q.shape[1], device=cuda_device)
    pre = 128 ** -0.5 * kernels.LOG2E
    want = ops.quant_pool(ops.gather_tiles(q, layout.perm, heads),
                          ops.gather_tiles(k, layout.perm, heads),
                          layout.valid_count, layout.n_video_tiles, pre)
    got = ops.quant_pool(q, k, layout.valid_count, layout.n_video_tiles, pre,
                         perm=layout.perm)
    for key in ('q_i8', 'q_scale', 'k_i8', 'k_scale', 'feats_q', 'feats_k'):
        assert torch.equal(got[key], want[key]), key


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
