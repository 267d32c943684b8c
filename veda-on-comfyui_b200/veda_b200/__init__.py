"""veda_b200: the Veda sparse-attention hot path for B200 (sm_100a).

A thin C ABI (include/veda_b200.h, built into libveda_b200.so by
`python -m veda_b200.build`) over hand-written CUDA kernels:

  quant_pool        INT8 quantisation of Q (per 128 rows) and K (per 64 rows)
                    fused with the predictor's TripPool features
  tile_logits       predictor projection and tile logits
  select            top-k key tiles straight into ascending index lists
  sparse_attention  block-sparse INT8 QK^T / 16-bit PV attention on tcgen05
                    tensor cores with TMEM accumulators, TMA tile loads

and, above it, the reference's interfaces for this path: the backend
contract (`backend.Backend`, `backend.create`), the kernel API
(`kernels.attend`), the selection and tiling rules, an engine fast path
(`engine.VedaAttention`) and head sharding across GPUs (`sharding`).
Nothing here has a CPU fallback.
"""

from . import _lib  # noqa: F401
from ._lib import DeviceStatusError, LibraryMissing, VedaError  # noqa: F401

__version__ = '0.1.0'
