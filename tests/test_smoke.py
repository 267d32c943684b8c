"""The build / smoke entry points the round-end checks call."""

import pytest


@pytest.mark.gpu
def test_graft_smoke(cuda_device):
    import __graft_entry__
    __graft_entry__.smoke()


def test_graft_build_loads_the_library():
    """build() compiles (nvcc needs no GPU) and loads the C ABI."""
    import shutil
    import __graft_entry__
    if shutil.which('nvcc') is None:
        pytest.skip('nvcc not on PATH')
    __graft_entry__.build()
