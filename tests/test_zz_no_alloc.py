"""veda_tile_logits_static, the entry point that allocates nothing (its
scratch is a fixed device array inside the library), called through the C
ABI and compared with veda_tile_logits on two calls in a row.

Named to be collected last: it must pass both alone and after every other
test has used the library on the same device.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

ROWS_LIMIT = 16384  # VEDA_STATIC_LOGITS_ROWS in include/veda_b200.h


def _inputs(device, heads, n_q, n_k, seed):
    g = torch.Generator().manual_seed(seed)
    feats_q = torch.randn(heads, n_q, 384, generator=g).to(device)
    feats_k = torch.randn(heads, n_k, 384, generator=g).to(device)
    proj = (torch.randn(2, heads, 384, 128, generator=g) * 0.02).to(
        torch.bfloat16).to(device)
    return feats_q, feats_k, proj[0].contiguous(), proj[1].contiguous()


def _with_workspace(lib, stream, feats_q, feats_k, pq, pk, logits):
    heads, n_q, _ = feats_q.shape
    n_k = feats_k.shape[1]
    workspace = torch.empty((n_q + n_k) * heads * 128, dtype=torch.float32,
                            device=feats_q.device)
    return lib.veda_tile_logits(feats_q.data_ptr(), feats_k.data_ptr(),
                                pq.data_ptr(), pk.data_ptr(), 0, heads, n_q,
                                n_k, workspace.data_ptr(), logits.data_ptr(),
                                stream)


def _static(lib, stream, feats_q, feats_k, pq, pk, logits):
    heads, n_q, _ = feats_q.shape
    n_k = feats_k.shape[1]
    return lib.veda_tile_logits_static(feats_q.data_ptr(), feats_k.data_ptr(),
                                       pq.data_ptr(), pk.data_ptr(), 0, heads,
                                       n_q, n_k, logits.data_ptr(), stream)


def test_static_scratch_logits_equal_the_workspace_entry_point(cuda_device):
    from veda_b200 import _lib
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    # cfg1's predictor shape (24 heads x 256 tiles), then a smaller one: the
    # second call must not see anything the first left in the scratch
    for heads, n_q, n_k, seed in [(24, 256, 256, 1), (3, 40, 72, 2)]:
        inputs = _inputs(cuda_device, heads, n_q, n_k, seed)
        want = torch.empty(heads, n_q, n_k, dtype=torch.float32,
                           device=cuda_device)
        got = torch.full_like(want, float('nan'))
        assert _with_workspace(lib, stream, *inputs, want) == 0, \
            lib.veda_last_error()
        # a first call loads the module (and its static array) if needed
        assert _static(lib, stream, *inputs, got) == 0, lib.veda_last_error()
        got.fill_(float('nan'))
        torch.cuda.synchronize(cuda_device)
        # free device memory as the driver sees it, so an allocation made
        # by the library itself (not only torch's) would show
        free_before, _ = torch.cuda.mem_get_info(cuda_device)
        assert _static(lib, stream, *inputs, got) == 0, lib.veda_last_error()
        torch.cuda.synchronize(cuda_device)
        free_after, _ = torch.cuda.mem_get_info(cuda_device)
        assert free_after == free_before
        assert torch.equal(got, want)


def test_static_scratch_rejects_oversize_calls(cuda_device):
    from veda_b200 import _lib
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    heads, n = 24, ROWS_LIMIT // 48 + 1        # (n + n) * 24 > the limit
    inputs = _inputs(cuda_device, 1, 1, 1, 3)  # valid pointers, never read
    logits = torch.empty(1, dtype=torch.float32, device=cuda_device)
    rc = lib.veda_tile_logits_static(*(t.data_ptr() for t in inputs), 0,
                                     heads, n, n, logits.data_ptr(), stream)
    assert rc == _lib.ERR_INVALID
    assert b'static scratch limit' in lib.veda_last_error()
