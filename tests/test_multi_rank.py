"""Head sharding on CPU with gloo (world size 2 and 4): the host-side logic
of the multi-GPU path, and a failed rank seen by its peers as an error.

Each rank runs a stand-in per-head attention (exact fp32 softmax attention
in torch on its head slice), the shards are all-gathered, and the assembled
output must equal the single-process result bit for bit.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _attention(q, k, v, scale_rows=None):
    s = torch.einsum('nhd,mhd->hnm', q.float(), k.float()) * q.shape[-1] ** -0.5
    if scale_rows is not None:
        s = s * scale_rows[:, None, None]
    return torch.einsum('hnm,mhd->nhd', torch.softmax(s, -1), v.float())


def _inputs():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(64, 8, 16, generator=g) for _ in range(3))
    return q, k, v, torch.rand(8, generator=g) + 0.5


def _worker(rank, world, port, queue):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from veda_b200 import sharding
        q, k, v, scale = _inputs()
        runner = sharding.HeadSharded(_attention)
        out = runner(q, k, v, head_args={'scale_rows': scale})
        lo, hi = sharding.head_range(8, rank, world)
        queue.put((rank, lo, hi, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 4])
def test_head_sharded_gather_equals_single_process(world):
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, scale = _inputs()
    want = _attention(q, k, v, scale)
    spans = sorted((lo, hi) for _, lo, hi, _ in results)
    assert spans == [(r * 8 // world, (r + 1) * 8 // world)
                     for r in range(world)]
    for _, _, _, out in results:
        assert torch.equal(out, want)


def _failing_worker(rank, world, port, queue):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    from veda_b200 import sharding

    def leave(message, code):
        queue.put((rank, message))
        queue.close()
        queue.join_thread()
        os._exit(code)

    if rank == 1:
        # this rank fails between steps: it never reaches the all-gather
        leave('raised', 3)
    try:
        sharding.gather_heads(torch.zeros(4, 2, 16))
        leave('no error', 0)
    except Exception as error:  # the peer's failure surfaces as an error
        leave(type(error).__name__, 0)


def test_a_failed_rank_is_an_error_for_its_peers_not_a_hang():
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, queue))
             for r in range(2)]
    for p in procs:
        p.start()
    got = dict(queue.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == 'raised'
    assert got[0] != 'no error'


def test_head_range_rules():
    from veda_b200 import sharding
    assert [sharding.head_range(24, r, 8) for r in range(8)][-1] == (21, 24)
    assert sharding.head_range(56, 3, 8) == (21, 28)
    with pytest.raises(ValueError):
        sharding.head_range(24, 0, 5)
    with pytest.raises(ValueError):
        sharding.head_range(24, 2, 2)
