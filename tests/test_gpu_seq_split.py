"""Sequence split over two GPUs (NCCL): the decode runtime with every
sequence's latents sharded over the ranks and the per-layer cross-GPU LSE
merge gives the logits of the unsplit runtime (2e-2 on bf16 logits).

Runs ``seq_split_ranks.py`` as two ranks through ``torch.distributed.run``;
skipped on a machine with one GPU.  The one-GPU parity of the same shard
decomposition (shards emulated as separate calls, merged by
``slimkv_merge_partials``) is in ``test_gpu_decode.py``.
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


def test_sequence_split_runtime_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    cmd = ['timeout', '-k', '30', '600', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node', '2', '--master-addr', '127.0.0.1', '--master-port', str(free_port()),
           os.path.join(HERE, 'seq_split_ranks.py')]
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', CUDA_VISIBLE_DEVICES=os.environ.get('CUDA_VISIBLE_DEVICES', '0,1'))
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert 'PASS' in proc.stdout
