"""Tensor-parallel decode over two GPUs (NCCL): projections and MLP split by
KV head, attention split by sequence, against the unsplit runtime (attention
rows 2e-3; logits within a few bf16 ulps, the fp32 partial sums of the
row-parallel projections being rounded once where the unsplit runtime rounds
each GEMM output), eager and graph-captured.

Runs ``tp_ranks.py`` as two ranks through ``torch.distributed.run``; skipped
on a machine with one GPU.  The exchanges themselves are checked on CPU
(``test_tensor_parallel_exchange.py``).
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_tensor_parallel_runtime_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    cmd = ['timeout', '-k', '30', '600', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node', '2', '--master-addr', '127.0.0.1', '--master-port', str(free_port()),
           os.path.join(HERE, 'tp_ranks.py')]
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', CUDA_VISIBLE_DEVICES=os.environ.get('CUDA_VISIBLE_DEVICES', '0,1'))
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert 'PASS' in proc.stdout
