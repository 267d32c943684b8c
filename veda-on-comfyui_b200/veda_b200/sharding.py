"""Head sharding of one Veda attention layer across the GPUs of a node.

Heads are independent all the way through the hot path (scores, selection,
quantisation scales, attention), so each rank (one process per GPU) takes a
contiguous block of heads, runs the whole call on it with no exchange, and
the only collective is an all-gather of the outputs over NVLink / NVSwitch
(NCCL, or gloo on CPU for tests). Q / K / V are assumed present on every
rank, as they are in a tensor-parallel DiT block.

The gathered buffer is [world, N, H_local, D]: rank r's heads at index r.
`assemble` turns it into [N, H, D] (one copy); consumers that take strided
input (the scatter back to sequence order) can read the buffer as is.

On GPUs joined by NVSwitch the exchange can be folded into the attention
kernel instead: `MulticastOutput` holds the full [N, H, D] output in
symmetric memory bound to a multicast object, each rank's kernel stores its
heads' rows once through the multicast address (veda_sparse_attention_
multicast), and one small collective orders the stores before any rank
reads the others' heads. No separate all-gather runs.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist


def head_range(heads: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of `rank`'s heads: contiguous and equal (the all-gather
    needs equal shards), so `world` must divide `heads`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} of {world}')
    if heads % world:
        raise ValueError(f'{heads} heads do not split evenly over {world} '
                         'ranks')
    per = heads // world
    return rank * per, (rank + 1) * per


def gather_heads(local: torch.Tensor, group=None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather [N, H_local, D] shards into [world, N, H_local, D]."""
    world = dist.get_world_size(group)
    local = local.contiguous()
    shape = (world,) + tuple(local.shape)
    if out is None:
        out = torch.empty(shape, dtype=local.dtype, device=local.device)
    # shards are concatenated along the first dimension of a flat view
    flat = out.view((world * local.shape[0],) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(flat, local, group=group)
    return out


def assemble(gathered: torch.Tensor) -> torch.Tensor:
    """[world, N, H_local, D] -> [N, world * H_local, D]."""
    world, n, h_local, d = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(n, world * h_local, d)


class HeadSharded:
    """Runs `attention(q, k, v, **kw)` on this rank's heads and gathers.

    Args:
        attention: A per-head-independent attention call taking [N, H', D]
            q / k / v slices (e.g. engine.VedaAttention(...).layer, with
            per-head extras such as scores sliced by `head_args`).
        group: Process group (default: the world).
    """

    def __init__(self, attention: Callable[..., torch.Tensor], group=None):
        self.attention = attention
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def __call__(self, q, k, v, head_args: dict | None = None,
                 contiguous: bool = True, **kwargs) -> torch.Tensor:
        lo, hi = head_range(q.shape[1], self.rank, self.world)
        sliced = {name: t[lo:hi] for name, t in (head_args or {}).items()}
        local = self.attention(q[:, lo:hi], k[:, lo:hi], v[:, lo:hi],
                               **sliced, **kwargs)
        gathered = gather_heads(local, self.group)
        return assemble(gathered) if contiguous else gathered


class MulticastOutput:
    """The full [N, H, D] output of a head-sharded call on every rank, written
    by the ranks' attention kernels through an NVSwitch multicast address.

    Args:
        shape: (N, H, D) of the full output.
        dtype, device: Of the output.
        group: Process group of the ranks (default: the world).

    Raises:
        RuntimeError: If the device or the group has no multicast support
            (use `gather_heads` there).
    """

    def __init__(self, shape, dtype: torch.dtype, device: torch.device,
                 group=None):
        import torch.distributed._symmetric_memory as symm
        self.group = group if group is not None else dist.group.WORLD
        if not self.supported(device):
            raise RuntimeError(f'{device} has no multicast support')
        self.full = symm.empty(*shape, dtype=dtype, device=device)
        self.handle = symm.rendezvous(self.full, self.group)
        self.mc_base = int(self.handle.multicast_ptr or 0)
        if not self.mc_base:
            raise RuntimeError('the group has no multicast object')
        self._flag = torch.zeros(1, dtype=torch.int32, device=device)

    @staticmethod
    def supported(device: torch.device) -> bool:
        """Whether `device` can bind multicast memory."""
        try:
            from torch._C._distributed_c10d import _SymmetricMemory
            from torch.distributed._symmetric_memory import DeviceType
            return bool(_SymmetricMemory.has_multicast_support(
                DeviceType.CUDA, torch.device(device).index or 0))
        except (ImportError, AttributeError, RuntimeError):
            return False

    def local_view(self, lo: int, hi: int) -> torch.Tensor:
        """This rank's heads [lo, hi) of the full buffer ([N, hi - lo, D],
        strided): the `out` of the multicast attention call."""
        return self.full[:, lo:hi]

    def multicast_address(self, view: torch.Tensor) -> int:
        """The multicast address of `view`'s first element."""
        return self.mc_base + (view.data_ptr() - self.full.data_ptr())

    def complete(self) -> torch.Tensor:
        """Orders every rank's multicast stores before later work on the
        current stream (a one-element all-reduce on the same stream), and
        returns the full output."""
        dist.all_reduce(self._flag, group=self.group)
        return self.full
