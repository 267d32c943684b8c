"""The drop-in boundary exercised through the reference's own code.

integration/b200_int8.py is loaded as `veda_comfy.backends.b200_int8` of the
unmodified reference package in baseline/_ref (git-ignored; these tests skip
when it is absent) and registered the way a maintainer would register it
(`_MODULES` and `candidates`, backends/__init__.py:36, 78-86). The
reference's own `resolve` then loads it and runs its own `base.self_test`
(backends/base.py:123-155) on this GPU, and the reference's validity checks
are shown to catch a backend that ignores the block mask.
"""

import importlib.util
import os
import sys

import pytest
import torch

import conftest

REF = os.path.join(conftest.REPO, 'baseline', '_ref')
ADAPTER = os.path.join(conftest.PACKAGE_ROOT, 'integration', 'b200_int8.py')


def _reference_backends():
    if not os.path.isdir(os.path.join(REF, 'veda_comfy')):
        pytest.skip('the reference package is not in baseline/_ref')
    if REF not in sys.path:
        sys.path.append(REF)
    try:
        from veda_comfy import backends
        from veda_comfy.backends import base
    except ImportError as e:
        pytest.skip(f'the reference package does not import: {e}')
    return backends, base


def _load_adapter():
    name = 'veda_comfy.backends.b200_int8'
    module = sys.modules.get(name)
    if module is None:
        spec = importlib.util.spec_from_file_location(name, ADAPTER)
        module = importlib.util.module_from_spec(spec)
        module.__package__ = 'veda_comfy.backends'
        sys.modules[name] = module
        spec.loader.exec_module(module)
    return module


def test_registry_offers_b200_first_on_sm100_only(registered):
    """The registration rule: sm_100 gets the B200 backend, every other
    device keeps the reference's own choice."""
    backends, _, _ = registered
    make = lambda cc, family: backends.hardware.DeviceInfo(
        'cuda', 0, 'gpu', cc, family, 'x', 'linux', 'x86_64', None, False,
        '12.8')
    assert backends.candidates(make((10, 0), 'sm100')) == ['b200-int8']
    assert backends.candidates(make((9, 0), 'sm90')) == ['triton-int8']


@pytest.fixture
def registered(monkeypatch):
    """The reference registry with the B200 backend first for sm_100."""
    backends, base = _reference_backends()
    adapter = _load_adapter()
    monkeypatch.setitem(backends._MODULES, 'b200-int8', 'b200_int8')
    plain = backends.candidates

    def candidates(info):
        if info.kind == 'cuda' and info.cc and info.cc[0] == 10 and \
                info.subtype != 'rocm':
            return ['b200-int8']
        return plain(info)

    monkeypatch.setattr(backends, 'candidates', candidates)
    backends.reset()
    yield backends, base, adapter
    backends.reset()


@pytest.mark.gpu
def test_reference_registry_resolves_and_self_tests_b200(registered,
                                                         cuda_device):
    backends, base, adapter = registered
    resolution = backends.resolve(cuda_device)
    assert resolution.backend is not None, resolution.report()
    assert resolution.attempts == [('b200-int8', 'ok')], resolution.report()
    assert isinstance(resolution.backend, adapter.B200Int8)
    # the reference's self-test in both input types it declares
    for dtype in resolution.backend.dtypes:
        base.self_test(resolution.backend, cuda_device, dtype)
    from veda_b200 import ops
    ops.check_status(cuda_device)


@pytest.mark.gpu
def test_reference_self_test_rejects_a_backend_that_ignores_the_mask(
        registered, cuda_device):
    """The check that protects users works on this kernel: the same B200
    backend given a full mask instead of the caller's fails it."""
    backends, base, adapter = registered
    good = adapter.create(backends.hardware.describe(cuda_device))

    class Dense(base.Backend):
        name, display = 'dense', 'dense'
        dtypes, tolerance = good.dtypes, good.tolerance

        def attend(self, q, k, v, block_mask, layout):
            full = torch.ones_like(block_mask) & layout.kv_ok
            return good.attend(q, k, v, full, layout)

    with pytest.raises(base.BackendUnavailable, match='ignores the block'):
        base.self_test(Dense(), cuda_device)


def test_adapter_reports_a_device_it_cannot_use(registered):
    """`create` turns an unsupported device into the reference's
    BackendUnavailable, with no library call (runs without a GPU)."""
    backends, base, adapter = registered
    info = backends.hardware.DeviceInfo(
        'cuda', 0, 'NVIDIA GeForce RTX 5090', (12, 0), 'sm120', 'rtx50',
        'linux', 'x86_64', None, False, '12.8')
    with pytest.raises(base.BackendUnavailable, match='sm_100'):
        adapter.create(info)
