"""CPU oracle for the Veda sparse-attention hot path: TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithm of each step of
the hot path (veda-sparse/Veda-on-ComfyUI 0.3.1, package `veda_comfy`):

  tiling.py     tile permutation and layout constants (core/tiling.py)
  selection.py  budgets, Bresenham extras, top-k selection, block mask,
                ascending index lists (core/selection.py)
  predictor.py  TripPool features and tile logits (core/predictor.py)
  int8.py       per-block INT8 quantisation and the INT8 block-sparse
                attention arithmetic (kernels/sage/sparse_int8.py)
  attention.py  exact fp32 masked block-sparse attention (core/reference.py)

Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of
`bench.py` may import it, and only as the checker or as the timed CPU
baseline. The product (`veda_b200`) never imports it and has no CPU
fallback.

Pinning: `tests/golden/make_golden.py` runs the reference's own code in a
container where it is importable (its torch core on CPU and its Triton
kernels under `TRITON_INTERPRET=1`) and commits the outputs as fixtures;
`tests/test_oracle_golden.py` checks this oracle against them.
"""
