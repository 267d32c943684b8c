"""The B200 backend as a module of the reference's backend package.

Copy this file to `veda_comfy/backends/b200_int8.py` and add 'b200-int8' to
that package's `_MODULES` and `candidates` (backends/__init__.py:36, 78-86);
the registry then loads it lazily through `create(info)` and validates it
with its own `base.self_test` (backends/base.py:123-155) before first use,
like any other backend.

The class only forwards: the work happens in `veda_b200.backend`, and its
two error types are translated into the reference's, so the node shows the
right message (`MissingDependency`: the user can fix it by building the
library; `BackendUnavailable`: this device cannot run it).
"""

import torch

from . import base


class B200Int8(base.Backend):
    """Forwards the reference's backend contract to veda_b200."""

    def __init__(self, impl):
        self._impl = impl
        self.name, self.display = impl.name, impl.display
        self.dtypes, self.tolerance = impl.dtypes, impl.tolerance

    def attend(self, q, k, v, block_mask, layout):
        return self._impl.attend(q, k, v, block_mask, layout)

    def warmup_note(self):
        return self._impl.warmup_note()

    def explain_failure(self, error):
        return self._impl.explain_failure(error)


def create(info) -> base.Backend:
    """The backend for the device `info` describes (hardware.DeviceInfo)."""
    if info.kind != 'cuda' or info.cc is None or info.cc[0] != 10:
        raise base.BackendUnavailable('b200-int8 needs an sm_100 GPU')
    try:
        from veda_b200 import backend as vb
    except ImportError as error:
        raise base.MissingDependency(
            f'veda_b200 is not importable ({error}): put '
            f'veda-on-comfyui_b200/ on sys.path') from error
    try:
        return B200Int8(vb.create(torch.device('cuda', info.index)))
    except vb.MissingDependency as error:
        raise base.MissingDependency(str(error)) from error
    except vb.BackendUnavailable as error:
        raise base.BackendUnavailable(str(error)) from error
