"""Generates the golden fixtures from the reference's own code.

    python tests/golden/make_golden.py --reference <checkout of
        veda-sparse/Veda-on-ComfyUI 0.3.1>

Runs where the reference is importable (it does not travel to GPU hosts):
its torch core on CPU (`core.tiling`, `core.selection`, `core.predictor`,
`core.reference`) and its Triton kernels (`kernels/sage/sparse_int8.py`)
under Triton's CPU interpreter (`TRITON_INTERPRET=1`). Inputs are
regenerated from seeds by `problems.py`; the fixtures hold the reference's
outputs and a sha256 of the inputs they were computed from.

Outputs (this directory): selection.npz, quant.npz, attention.npz,
predictor.npz, meta.json.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

os.environ['TRITON_INTERPRET'] = '1'

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import problems  # noqa: E402
from oracle import selection as osel  # noqa: E402

# Rows of the large attention outputs kept in the fixtures.
ROW_STRIDE = {'selftest': 1, 'cfg0': 8, 'gpu_problem': 16}


def ref_budget(rsel, b: osel.Budget):
    return rsel.Budget(ratio=b.ratio) if b.tiles is None else rsel.Budget(
        tiles=b.tiles)


def ref_layout(rtil, case: problems.Case):
    if case.spans is None:
        real = case.seq_len if case.real is None else case.real
        spans = [rtil.TiledSpan(0, (1, 1, real), rtil.TileShape(1, 1, 128))]
        return rtil.build_tile_layout(spans, real)
    spans = [rtil.TiledSpan(s, g, rtil.TileShape(*t))
             for s, g, t in case.spans]
    return rtil.build_tile_layout(spans, case.seq_len)


def ref_mask(ref, case, scores, layout):
    rsel = ref['selection']
    blocks = rsel.column_blocks(layout, ref_budget(rsel, case.generated),
                                ref_budget(rsel, case.reference))
    index, keep = rsel.select(torch.from_numpy(scores), layout, blocks)
    return rsel.block_mask(index, keep, layout) & layout.kv_ok


def gen_selection(ref, meta, out):
    rsel = ref['selection']
    for name, case in problems.CASES.items():
        t0 = time.time()
        layout = ref_layout(ref['tiling'], case)
        ours = case.layout()
        assert np.array_equal(layout.perm.numpy(), ours.perm), name
        assert np.array_equal(layout.valid_count.numpy(), ours.valid_count)
        scores = problems.make_scores(case)
        mask = ref_mask(ref, case, scores, layout)
        index, count = rsel.tile_index_list(mask)
        # the oracle's list form of the reference's own mask
        o_index, o_count = osel.tile_index_list(mask.numpy())
        assert np.array_equal(o_count, count.numpy())
        live = np.arange(o_index.shape[-1]) < o_count[..., None]
        assert np.array_equal(np.where(live, o_index, -1),
                              np.where(live, index.numpy(), -1)), name
        blocks = case.blocks(ours)
        o_mask = osel.block_mask(osel.select_keep(scores, ours, blocks),
                                 ours) & ours.kv_ok[None, None, :]
        same = ~(o_mask != mask.numpy()).any(-1)
        tie_rows = np.zeros(same.shape, dtype=bool)
        tie_rows[:, :ours.n_video_tiles] = osel.boundary_ties(scores, ours,
                                                             blocks)
        out[f'{name}.mask_bits'] = np.packbits(mask.numpy(), axis=-1)
        out[f'{name}.count'] = count.numpy().astype(np.int16)
        meta['selection'][name] = {
            'scores_sha256': problems.sha256(scores),
            'n_tiles': ours.n_tiles, 'n_video_tiles': ours.n_video_tiles,
            'width': int(index.shape[-1]),
            'oracle_rows_differing': int((~same).sum()),
            'oracle_rows_differing_outside_ties': int((~same & ~tie_rows)
                                                      .sum()),
            'boundary_tie_rows': int(tie_rows.sum()),
        }
        print(f'selection {name}: {meta["selection"][name]} '
              f'({time.time() - t0:.1f}s)')


def gen_budgets(ref, meta):
    rsel = ref['selection']
    table = []
    for budget in [0.2, 1.0, 2.3, 2.5, 5.5, 12.0, 25.6, 26.0, 54.1, 102.4,
                   0.225, 3.999999999999]:
        for n_cols in [1, 4, 10, 72, 256, 594, 1024]:
            table.append([budget, n_cols, list(rsel.split_budget(budget,
                                                                 n_cols))])
    ratios = []
    for ratio in [0.1, 0.15, 0.2, 0.3, 1.0]:
        for real, n_cols in [(32760, 256), (320, 4), (4096, 32),
                             (131072, 1024), (2688, 24), (384, 4)]:
            b = rsel.Budget(ratio=ratio)
            ratios.append([ratio, real, n_cols, b.per_row(real, n_cols)])
    bres = {}
    for n_rows, frac in [(1000, 0.3), (256, 0.6), (594, 0.1), (72, 0.5),
                         (1024, 0.4), (192, 0.0), (37, 0.999999999999)]:
        bits = rsel.bresenham_extra(n_rows, frac, 'cpu').numpy()
        bres[f'{n_rows}:{frac!r}'] = np.packbits(bits).tolist()
    meta['budgets'] = {'split_budget': table, 'per_row': ratios,
                       'bresenham_packbits': bres}


def gen_quant(ref, meta, out):
    si = ref['sparse_int8']
    x = problems.quant_input()
    pre = 128 ** -0.5 * si.LOG2E
    qi, qs = si.quantize(x, si.TILE, pre_scale=pre)
    ki, ks = si.quantize(x, si.KEY_BLOCK)
    out['q_int8'], out['q_scale'] = qi.numpy(), qs.numpy()
    out['k_int8'], out['k_scale'] = ki.numpy(), ks.numpy()
    meta['quant'] = {'input_sha256': problems.sha256(x), 'pre_scale': pre}


def ref_int8_attend(ref, q, k, v, mask, layout):
    """The reference INT8 path, `sparse_int8.attend` minus its device
    capability query (the interpreter has no device), i.e. the pointer
    kernel it runs by default (USE_TMA = False)."""
    si, rsel = ref['sparse_int8'], ref['selection']
    index, count = rsel.tile_index_list(mask & layout.kv_ok)
    slots, heads, dim = q.shape
    q8, qs = si.quantize(q, si.TILE, pre_scale=dim ** -0.5 * si.LOG2E)
    k8, ks = si.quantize(k, si.KEY_BLOCK)
    blocks, bcount, valid = si.key_blocks(index, count, layout.valid_count,
                                          si.KEY_BLOCK)
    v16 = v.to(torch.float16)
    out = torch.empty_like(q)
    si._attention_kernel[(slots // si.TILE, heads)](
        q8, k8, v16, qs, ks, blocks, bcount, valid, out,
        q.stride(0), q.stride(1), v16.stride(0), v16.stride(1),
        qs.stride(0), ks.stride(0), blocks.stride(0), blocks.stride(1),
        n_q_tiles=slots // si.TILE, D=dim, BLK=si.KEY_BLOCK,
        BLOCK_M=si.TILE)
    return out


def gen_attention(ref, meta, out):
    rref = ref['reference']
    for name in ['selftest', 'cfg0', 'gpu_problem']:
        t0 = time.time()
        case = problems.CASES[name]
        q, k, v, scores, _ = problems.make_problem(case)
        layout = ref_layout(ref['tiling'], case)
        mask = ref_mask(ref, case, scores, layout)
        int8_out = ref_int8_attend(ref, q, k, v, mask, layout)
        fp32_out = torch.cat([
            rref.block_sparse_attention(
                q[:, h:h + 1].float(), k[:, h:h + 1].float(),
                v[:, h:h + 1].float(), mask[h:h + 1], layout)
            for h in range(case.heads)], dim=1)
        stride = ROW_STRIDE[name]
        rows = np.arange(0, q.shape[0], stride)
        out[f'{name}.rows'] = rows.astype(np.int32)
        out[f'{name}.int8_out'] = int8_out[rows].float().numpy().astype(
            np.float16)
        out[f'{name}.fp32_out'] = fp32_out[rows].float().numpy().astype(
            np.float16)
        meta['attention'][name] = {
            'qkv_sha256': problems.sha256(q, k, v),
            'scores_sha256': problems.sha256(scores),
            'row_stride': stride}
        print(f'attention {name}: {time.time() - t0:.1f}s')


def gen_predictor(ref, meta, out):
    rpred = ref['predictor']
    for name in ['selftest', 'gpu_problem']:
        case = problems.CASES[name]
        q, k, _, _, _ = problems.make_problem(case)
        layout = ref_layout(ref['tiling'], case)
        proj = problems.make_proj(case)
        fq = rpred.pool_video_tiles(q, layout)
        fk = rpred.pool_video_tiles(k, layout)
        logits = rpred.tile_logits(fq, fk, proj[0], proj[1])
        out[f'{name}.feats_q'] = fq.numpy()
        out[f'{name}.feats_k'] = fk.numpy()
        out[f'{name}.logits'] = logits.numpy()
        meta.setdefault('predictor', {})[name] = {
            'proj_sha256': problems.sha256(proj),
            'qk_sha256': problems.sha256(q, k)}


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--reference', required=True)
    parser.add_argument('--only', default='')
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    from veda_comfy.core import predictor, reference, selection, tiling
    from veda_comfy.kernels.sage import sparse_int8
    ref = dict(selection=selection, tiling=tiling, predictor=predictor,
               reference=reference, sparse_int8=sparse_int8)
    meta_path = os.path.join(HERE, 'meta.json')
    meta = (json.load(open(meta_path)) if os.path.exists(meta_path)
            else {})
    meta.setdefault('selection', {})
    meta.setdefault('attention', {})
    meta['torch'] = torch.__version__
    parts = args.only.split(',') if args.only else [
        'selection', 'budgets', 'quant', 'attention', 'predictor']
    if 'selection' in parts:
        out = {}
        gen_selection(ref, meta, out)
        np.savez_compressed(os.path.join(HERE, 'selection.npz'), **out)
    if 'budgets' in parts:
        gen_budgets(ref, meta)
    if 'quant' in parts:
        out = {}
        gen_quant(ref, meta, out)
        np.savez_compressed(os.path.join(HERE, 'quant.npz'), **out)
    if 'predictor' in parts:
        out = {}
        gen_predictor(ref, meta, out)
        np.savez_compressed(os.path.join(HERE, 'predictor.npz'), **out)
    if 'attention' in parts:
        out = {}
        gen_attention(ref, meta, out)
        np.savez_compressed(os.path.join(HERE, 'attention.npz'), **out)
    with open(meta_path, 'w') as f:
        json.dump(meta, f, indent=1, sort_keys=True)


if __name__ == '__main__':
    main()
