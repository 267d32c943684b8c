"""bench.py host logic that needs no GPU: the reference GPU arm's package
lookup, and the layouts it builds for each config, which must be this
build's layouts (same permutation, same tile counts), so both arms time the
same work."""


import numpy as np
import pytest

import conftest  # noqa: F401  (puts the repository on sys.path)

# (spans, seq_len, real rows) of configs 1-4, as bench.config_workload
# builds them
CONFIGS = {
    'cfg1': (None, 32768, 32760),
    'cfg3_16k': (None, 16384, 16384),
    'cfg3_128k': (None, 131072, 131072),
    'cfg4': ([(8192, (1, 1, 24576), (1, 1, 128))], 32768, 32768),
}


def _bench():
    import bench
    return bench


def test_reference_gpu_arm_reports_a_missing_package(monkeypatch, tmp_path):
    bench = _bench()
    monkeypatch.setattr(bench, 'REF_PACKAGE', str(tmp_path / 'absent'))
    mods, why = bench._reference_gpu_modules()
    assert mods is None
    assert 'baseline/_ref' in why


@pytest.mark.parametrize('name', sorted(CONFIGS))
def test_reference_arm_layouts_match_this_build(name):
    bench = _bench()
    mods, why = bench._reference_gpu_modules()
    if mods is None:
        pytest.skip(why)
    _, rtil, _ = mods
    from veda_b200 import tiling
    spans, seq, real = CONFIGS[name]
    ref = bench.reference_layout(rtil, spans, seq, real, 'cpu')
    if spans is None:
        ours = tiling.identity_layout(real, 'cpu')
    else:
        ours = tiling.build_tile_layout(
            [tiling.TiledSpan(st, g, tiling.TileShape(*t))
             for st, g, t in spans], seq, 'cpu')
    assert np.array_equal(np.asarray(ours.perm.cpu()),
                          ref.perm.cpu().numpy())
    assert ours.n_video_tiles == ref.n_video_tiles
    assert ours.n_tiles == ref.n_tiles
    assert np.array_equal(ours.valid_count.cpu().numpy(),
                          ref.valid_count.cpu().numpy())
