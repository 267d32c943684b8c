"""Head sharding on two GPUs with the output exchanged by the attention
kernel's multicast stores (torchrun, NCCL). Skipped below two GPUs."""

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_multicast_output_equals_nccl_all_gather():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    env = dict(os.environ, NCCL_DEBUG='WARN')
    cmd = ['timeout', '-k', '30', '300', sys.executable, '-m',
           'torch.distributed.run', '--nnodes=1', '--nproc-per-node', '2',
           '--master-addr', '127.0.0.1', '--master-port', str(_port()),
           os.path.join(HERE, 'multi_gpu_worker.py')]
    run = subprocess.run(cmd, capture_output=True, text=True, env=env)
    out = run.stdout + run.stderr
    if 'SKIP no multicast support' in out:
        pytest.skip('no multicast support on this node')
    assert run.returncode == 0, out[-4000:]
