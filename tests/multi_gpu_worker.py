"""One rank of the 2-GPU multicast-output check (run by torchrun from
tests/test_multi_gpu.py): a head-sharded layer with the output exchanged
through the attention kernel's multicast stores must equal, bit for bit,
an NCCL all-gather of the plain kernel's per-rank outputs, and the oracle
on sampled rows."""

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.dirname(HERE),
                os.path.join(os.path.dirname(HERE), 'veda-on-comfyui_b200'),
                HERE, os.path.join(HERE, 'golden')]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    rank = int(os.environ['RANK'])
    world = int(os.environ['WORLD_SIZE'])
    device = torch.device('cuda', int(os.environ['LOCAL_RANK']))
    torch.cuda.set_device(device)
    dist.init_process_group('nccl', device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import helpers
        import problems
        from oracle import int8 as oint8
        from veda_b200 import kernels, ops, selection, sharding
        case = problems.CASES['cfg0']
        q, k, v, scores, olayout = problems.make_problem(case)
        heads = case.heads
        lo, hi = sharding.head_range(heads, rank, world)
        layout = helpers.device_layout(case, device)
        blocks = helpers.product_blocks(case, layout)
        index, count = selection.select_index(
            torch.from_numpy(scores[lo:hi]).to(device), layout, blocks)
        dq, dk, dv = (t[:, lo:hi].contiguous().to(device) for t in (q, k, v))
        quant = ops.quant_pool(dq, dk, layout.valid_count, 0,
                               128 ** -0.5 * kernels.LOG2E, pool=False)
        args = (quant['q_i8'], quant['q_scale'], quant['k_i8'],
                quant['k_scale'], dv, index, count, layout.valid_count)
        if not sharding.MulticastOutput.supported(device):
            print('SKIP no multicast support', flush=True)
            return 0
        mc = sharding.MulticastOutput(tuple(q.shape), torch.bfloat16, device)
        view = mc.local_view(lo, hi)
        ops.sparse_attention(*args, out=view,
                             out_multicast=mc.multicast_address(view))
        full = mc.complete().clone()
        ops.check_status(device)
        plain = ops.sparse_attention(*args)
        want = sharding.assemble(sharding.gather_heads(plain))
        same = bool(torch.equal(full, want))
        # sampled rows of this rank's heads against the oracle
        gidx = np.zeros((heads,) + tuple(index.shape[1:]), np.int32)
        gcnt = np.zeros((heads, index.shape[1]), np.int32)
        gidx[lo:hi] = index.cpu().numpy()
        gcnt[lo:hi] = count.cpu().numpy()
        ref = oint8.int8_block_sparse(
            q.float().numpy(), k.float().numpy(), v.float().numpy(), gidx,
            gcnt, olayout.valid_count, heads=range(lo, hi), q_tiles=[0, 31])
        rows = np.r_[0:128, 31 * 128:32 * 128]
        m = helpers.compare(full[rows][:, lo:hi].float().cpu().numpy(),
                            ref[rows][:, lo:hi])
        ok = same and helpers.within_int8_tolerance(m)
        print(f'rank {rank}: equal={same} oracle={m}', flush=True)
        flag = torch.tensor([1 if ok else 0], device=device)
        dist.all_reduce(flag, dist.ReduceOp.MIN)
        return 0 if flag.item() == 1 else 1
    finally:
        dist.destroy_process_group()


if __name__ == '__main__':
    sys.exit(main())
