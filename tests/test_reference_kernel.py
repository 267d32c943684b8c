"""Parity with the reference's own Triton INT8 kernel run on the same GPU:
`veda_comfy.kernels.sage.sparse_int8.attend` from the unmodified reference
package, when it has been placed in baseline/_ref (git-ignored; the tests
skip when it is absent), against this build's `kernels.attend` on the same
inputs and index lists.

The reference rounds P and V to fp16 and sums P V per 64-key block in
fp16; this build keeps P in the input's 16-bit type and accumulates in
fp32, so the bar is the attention tolerance (cos >= 0.9995, max |diff|
<= 2e-2 at unit scale), not bit equality.
"""

import os
import sys

import pytest
import torch

import conftest
import helpers
import problems

pytestmark = pytest.mark.gpu

REF = os.path.join(conftest.REPO, 'baseline', '_ref')


def _reference():
    if not os.path.isdir(os.path.join(REF, 'veda_comfy')):
        pytest.skip('the reference package is not in baseline/_ref')
    if REF not in sys.path:
        sys.path.append(REF)
    try:
        from veda_comfy.kernels.sage import sparse_int8
    except ImportError as e:
        pytest.skip(f'the reference package does not import: {e}')
    return sparse_int8


@pytest.mark.parametrize('name', ['gpu_problem', 'cfg1'])
@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
def test_attention_matches_reference_triton_kernel(cuda_device, name, dtype):
    ref = _reference()
    from veda_b200 import kernels
    from veda_b200 import selection as vs
    case = problems.CASES[name]
    q, k, v, scores, olayout = problems.make_problem(case)
    heads = min(case.heads, 4)  # four heads keep the cfg1 case quick
    q, k, v = (t[:, :heads].to(dtype).contiguous().to(cuda_device)
               for t in (q, k, v))
    layout = helpers.device_layout(case, cuda_device)
    index, count = vs.select_index(
        torch.from_numpy(scores[:heads]).to(cuda_device), layout,
        helpers.product_blocks(case, layout))
    want = ref.attend(q, k, v, index, count, layout.valid_count)
    got = kernels.attend(q, k, v, index, count, layout.valid_count)
    real = torch.from_numpy(olayout.slot_valid.astype(bool)).to(cuda_device)
    m = helpers.compare(got[real].float().cpu().numpy(),
                        want[real].float().cpu().numpy())
    assert helpers.within_int8_tolerance(m), m
