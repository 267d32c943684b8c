"""The C ABI (include/veda_b200.h) on CPU: the library loads, exports every
declared entry point, and the ctypes signatures in `veda_b200._lib` agree
with the header argument for argument. No kernel is launched.

The library is built in-tree first if it is missing (nvcc cross-compiles
for sm_100a without a GPU).
"""

import ctypes
import os
import re
import shutil
import subprocess

import pytest

import conftest

HEADER = os.path.join(conftest.REPO, 'include', 'veda_b200.h')

_DECL = re.compile(r'^(int|const char\s*\*)\s*(veda_\w+)\s*\(([^)]*)\)\s*;',
                   re.MULTILINE)


def _declarations() -> dict:
    with open(HEADER) as f:
        text = re.sub(r'/\*.*?\*/', '', f.read(), flags=re.DOTALL)
    decls = {}
    for ret, name, args in _DECL.findall(text):
        args = ' '.join(args.split())
        params = [] if args in ('', 'void') else [
            a.strip() for a in args.split(',')]
        decls[name] = (ret.replace(' ', ''), params)
    return decls


def _ctype(param: str):
    from veda_b200 import _lib
    if '*' in param:
        if 'veda_column_block' in param:
            return ctypes.POINTER(_lib.ColumnBlock)
        return ctypes.c_void_p
    kind = param.rsplit(' ', 1)[0].replace('const ', '').strip()
    return {'int': ctypes.c_int, 'int64_t': ctypes.c_int64,
            'uint64_t': ctypes.c_uint64, 'float': ctypes.c_float}[kind]


@pytest.fixture(scope='module')
def lib():
    from veda_b200 import _lib, build
    if not os.path.exists(_lib.LIBRARY):
        if shutil.which('nvcc') is None and not os.path.exists(
                '/usr/local/cuda/bin/nvcc'):
            pytest.fail('libveda_b200.so is missing and nvcc is not found')
        build.build()
    return _lib.load()


def test_header_declares_the_entry_points():
    decls = _declarations()
    assert {'veda_quant_pool', 'veda_select', 'veda_sparse_attention',
            'veda_tile_logits', 'veda_mask_to_index', 'veda_quantize',
            'veda_gather_tiles', 'veda_scatter_tiles', 'veda_abi_version',
            'veda_last_error', 'veda_device_supported'} <= set(decls)


def test_ctypes_signatures_match_the_header():
    from veda_b200 import _lib
    decls = _declarations()
    assert set(decls) == set(_lib.SIGNATURES)
    for name, (ret, params) in decls.items():
        want = [_ctype(p) for p in params]
        got = _lib.SIGNATURES[name]
        assert len(got) == len(want), name
        for i, (g, w) in enumerate(zip(got, want)):
            assert g == w, f'{name} argument {i}: {g} vs {w} ({params[i]})'


def test_every_declared_symbol_is_exported(lib):
    for name in _declarations():
        assert hasattr(lib, name), name
    nm = shutil.which('nm')
    if nm:
        from veda_b200 import _lib
        out = subprocess.run([nm, '-D', '--defined-only', _lib.LIBRARY],
                             capture_output=True, text=True, check=True)
        exported = {line.split()[-1] for line in out.stdout.splitlines()
                    if line.strip()}
        assert set(_declarations()) <= exported


def test_version_and_error_calls_need_no_gpu(lib):
    with open(HEADER) as f:
        version = int(re.search(r'#define VEDA_ABI_VERSION (\d+)',
                                f.read()).group(1))
    assert lib.veda_abi_version() == version
    assert isinstance(lib.veda_last_error(), bytes)
    import torch
    if not torch.cuda.is_available():
        assert lib.veda_device_supported(0) == 0


def test_library_is_sm100a_only():
    """The build flags name one target, sm_100a, and no PTX fallback."""
    from veda_b200 import build
    assert build.ARCH == ['-gencode', 'arch=compute_100a,code=sm_100a']


def test_static_logits_rejects_oversize_sizes_before_any_device_work():
    """veda_tile_logits_static checks its sizes before it looks at a device,
    with 64-bit arithmetic: n_q = n_k = 2^30 (whose int sum overflows) is
    refused with VEDA_ERR_INVALID here, on a machine with no GPU at all.
    The pointers are never dereferenced."""
    from veda_b200 import _lib
    lib = _lib.load()
    fake = ctypes.c_void_p(256)
    for heads, n_q, n_k in [(1, 2 ** 30, 2 ** 30), (1, 20000, 1),
                            (24, 256, 512), (65535, 1, 1)]:
        rc = lib.veda_tile_logits_static(fake, fake, fake, fake, _lib.BF16,
                                         heads, n_q, n_k, fake, None)
        assert rc == _lib.ERR_INVALID, (heads, n_q, n_k, rc)
        assert b'static scratch limit' in lib.veda_last_error()
