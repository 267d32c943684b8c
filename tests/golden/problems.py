"""Seeded synthetic problems shared by the golden-fixture generator and the
tests. Inputs are regenerated from seeds with torch's CPU generator (the
same draws on every machine with the same torch), so fixtures only store
expected outputs and a sha256 of the regenerated inputs.

Shapes follow the benchmark configs and the reference's own test problems:
  * selftest     veda_comfy/backends/base.py:94-120 (text 70 | history
                 1x8x16 | audio 40 | target 5x8x8 tiled 4x4x8; 2 heads;
                 x ~ 1.5 N(0,1); scores N(0,1); budgets 2 / 1 tiles)
  * gpu_problem  tests/gpu/test_gpu_backends.py:51-70 (S=6000, 4 heads,
                 reference 1x16x24 tiled 1x8x16, target 7x16x24 tiled
                 4x4x8; budgets ratio 0.1 / 0.2)
  * cfg0..cfg4   the synthetic benchmark configs (identity tile order:
                 one 1 x 1 x L span tiled 1 x 1 x 128).
"""

from __future__ import annotations

import dataclasses
import hashlib

import numpy as np
import torch

from oracle import selection as osel
from oracle import tiling as otil

HEAD_DIM = 128


@dataclasses.dataclass(frozen=True)
class Case:
    name: str
    heads: int
    seq_len: int
    spans: tuple | None = None       # None: identity layout over `real`
    real: int | None = None
    seed: int = 0
    x_scale: float = 1.0
    k_offset: float = 0.0            # sigma of a per-(head, channel) K offset
    scores: str = 'rand'             # 'rand' U(0,1), 'randn', 'levels'
    shared_stream: bool = False      # scores drawn after q/k/v, same stream
    qkv_draw: str = 'separate'       # 'separate': 3 calls; 'stacked': 1 call
    generated: osel.Budget = osel.Budget(tiles=4)
    reference: osel.Budget = osel.Budget(ratio=1.0)

    def layout(self) -> otil.Layout:
        if self.spans is None:
            return otil.identity_layout(self.seq_len, self.real)
        return otil.build_tile_layout(list(self.spans), self.seq_len)

    def blocks(self, layout=None):
        layout = self.layout() if layout is None else layout
        return osel.column_blocks(layout, self.generated, self.reference)


_SELFTEST_SPANS = ((70, (1, 8, 16), (1, 8, 16)), (238, (5, 8, 8), (4, 4, 8)))
_GPU_SPANS = ((300, (1, 16, 24), (1, 8, 16)), (1000, (7, 16, 24), (4, 4, 8)))

CASES = {c.name: c for c in [
    Case('selftest', heads=2, seq_len=558, spans=_SELFTEST_SPANS,
         x_scale=1.5, scores='randn', shared_stream=True,
         qkv_draw='stacked', generated=osel.Budget(tiles=2),
         reference=osel.Budget(tiles=1)),
    Case('gpu_problem', heads=4, seq_len=6000, spans=_GPU_SPANS,
         scores='randn', shared_stream=True,
         generated=osel.Budget(ratio=0.1), reference=osel.Budget(ratio=0.2)),
    Case('cfg0', heads=4, seq_len=4096, seed=100,
         generated=osel.Budget(tiles=4)),
    Case('cfg1', heads=24, seq_len=32768, real=32760, seed=101,
         k_offset=2.0, generated=osel.Budget(tiles=26)),
    Case('cfg1_sp90', heads=24, seq_len=32768, real=32760, seed=101,
         k_offset=2.0, generated=osel.Budget.sparsity(90)),
    Case('cfg3_16k', heads=24, seq_len=16384, seed=103,
         generated=osel.Budget.sparsity(90)),
    Case('cfg3_131k', heads=2, seq_len=131072, seed=104,
         generated=osel.Budget.sparsity(90)),
    Case('cfg4', heads=24, seq_len=32768,
         spans=((8192, (1, 1, 24576), (1, 1, 128)),), seed=105,
         generated=osel.Budget(tiles=32)),
    Case('refblock', heads=3, seq_len=3400,
         spans=((0, (2, 16, 16), (1, 8, 16)), (600, (9, 12, 20), (2, 8, 8))),
         seed=106, scores='randn', generated=osel.Budget(ratio=0.15),
         reference=osel.Budget(ratio=0.3)),
    Case('keepall', heads=2, seq_len=1200,
         spans=((40, (3, 8, 24), (2, 8, 8)),), seed=107,
         generated=osel.Budget(ratio=1.0)),
    Case('frac_tiles', heads=3, seq_len=8192, real=8000, seed=108,
         generated=osel.Budget(tiles=2.3)),
    Case('ties', heads=4, seq_len=8192, seed=109, scores='levels',
         generated=osel.Budget(tiles=7)),
]}


def _score_draw(case: Case, n: int, gen: torch.Generator) -> torch.Tensor:
    shape = (case.heads, n, n)
    if case.scores == 'rand':
        return torch.rand(shape, generator=gen)
    if case.scores == 'randn':
        return torch.randn(shape, generator=gen)
    if case.scores == 'levels':
        return torch.floor(torch.rand(shape, generator=gen) * 8.0) / 8.0
    raise ValueError(case.scores)


def packed_qkv(case: Case, gen: torch.Generator):
    """q, k, v [S, H, D] bf16 in packed (sequence) order."""
    shape = (case.seq_len, case.heads, HEAD_DIM)
    if case.qkv_draw == 'stacked':
        x = torch.randn((3,) + shape, generator=gen) * case.x_scale
        q, k, v = x[0], x[1], x[2]
    else:
        q, k, v = (torch.randn(shape, generator=gen) * case.x_scale
                   for _ in range(3))
    if case.k_offset:
        k = k + torch.randn(case.heads, HEAD_DIM, generator=gen) * \
            case.k_offset
    return tuple(t.to(torch.bfloat16) for t in (q, k, v))


def make_scores(case: Case) -> np.ndarray:
    """[H, n_video, n_video] fp32 scores of a case."""
    layout = case.layout()
    if case.shared_stream:
        gen = torch.Generator().manual_seed(case.seed)
        packed_qkv(case, gen)
    else:
        gen = torch.Generator().manual_seed(case.seed + 1000)
    return _score_draw(case, layout.n_video_tiles, gen).numpy()


def make_problem(case: Case):
    """(q, k, v tile-ordered bf16 torch tensors [N, H, D], scores, layout)."""
    layout = case.layout()
    gen = torch.Generator().manual_seed(case.seed)
    packed = packed_qkv(case, gen)
    if case.shared_stream:
        scores = _score_draw(case, layout.n_video_tiles, gen).numpy()
    else:
        scores = make_scores(case)
    perm = torch.from_numpy(layout.perm)
    pad = perm < 0
    tiled = []
    for x in packed:
        t = x[perm.clamp(min=0)].clone()
        t[pad] = 0
        tiled.append(t)
    return tiled[0], tiled[1], tiled[2], scores, layout


def make_proj(case: Case, seed: int = 55) -> torch.Tensor:
    """[2, H, 3D, D] bf16 predictor projections (q, k) drawn like the
    reference's synthetic bundles (random x 0.02, tests/veda_testing.py)."""
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(2, case.heads, 3 * HEAD_DIM, HEAD_DIM, generator=gen)
            * 0.02).to(torch.bfloat16)


def sha256(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = a.contiguous().view(torch.uint8).numpy() if a.dtype in (
                torch.bfloat16,) else a.contiguous().numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def quant_input(seed: int = 7) -> torch.Tensor:
    """[512, 3, 128] bf16 with an all-zero (block, head), a large-magnitude
    head and exact .5 quantisation boundaries planted."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(512, 3, HEAD_DIM, generator=gen)
    x[128:256, 1] = 0.0
    x[:, 2] *= 40.0
    x[0, 0, :4] = torch.tensor([127.0, -63.5, 0.5, -0.5]) / 127.0 * 3.0
    return x.to(torch.bfloat16)
