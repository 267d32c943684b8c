"""Test setup: import paths, the `gpu` marker, shared fixtures.

`-m "not gpu"` runs on any machine: the oracle against the golden fixtures
(made from the reference's own code), the host-side logic, and the C ABI's
loading and symbol table. `-m gpu` runs the CUDA kernels through the C ABI
against the oracle and the fixtures on a B200.
"""

import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PACKAGE_ROOT = os.path.join(REPO, 'veda-on-comfyui_b200')
for path in (REPO, PACKAGE_ROOT, os.path.join(HERE, 'golden')):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line(
        'markers', 'gpu: needs an sm_100 GPU and the built CUDA library')


@pytest.fixture(scope='session')
def cuda_device():
    """The sm_100 device the GPU tests run on; a GPU test fails loudly when
    the CUDA library is missing rather than skipping to a fallback."""
    import torch
    from veda_b200 import _lib
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    lib = _lib.load()  # raises LibraryMissing: the build is part of the test
    device = torch.device('cuda', torch.cuda.current_device())
    assert lib.veda_device_supported(device.index) == 1, \
        f'{torch.cuda.get_device_name(device)} is not sm_100'
    return device


@pytest.fixture(autouse=True)
def _check_device_status(request):
    """After every GPU test, the device status word must be clean."""
    yield
    if request.node.get_closest_marker('gpu') is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from veda_b200 import ops
    if getattr(request.node, 'expects_device_error', False):
        return
    ops.check_status(torch.device('cuda', torch.cuda.current_device()))
