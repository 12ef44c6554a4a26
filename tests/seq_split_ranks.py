"""Ranks of the two-GPU sequence-split check (launched by
``test_gpu_seq_split.py`` through ``torch.distributed.run``).

Every rank builds the same unsplit decode runtime (same seeds, so the same
weights and caches on every GPU) and a sequence-split runtime over the NCCL
group, copies its shard of the unsplit caches into the split runtime, then
decodes the same tokens with both: eagerly, then through CUDA graphs that
hold the NCCL all-gathers.  Logits must agree within the 2e-2 bar on bf16
logits; rank 0 prints PASS.
"""
import dataclasses
import gc
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from slimkv_b200.runtime import LatentDecodeRuntime, LatentLlamaConfig, RandomWeights, qwen25_14b_r2  # noqa: E402


def copy_shard(full, split):
    """This rank's latent rows (and, on the last rank, the raw caches) of the
    unsplit runtime's caches into the split runtime's."""
    sp = split.split
    offsets, rows = sp['offset'].tolist(), sp['rows'].tolist()
    for cf, cs in zip(full.caches, split.caches):
        for b, (off, n) in enumerate(zip(offsets, rows)):
            if sp['last']:
                n = min(cs['lat'].shape[1], cf['lat'].shape[1] - off)
            cs['lat'][b, :n].copy_(cf['lat'][b, off:off + n])
        if sp['last']:
            for key in ('raw_k_rot', 'raw_v'):
                cs[key].copy_(cf[key])
            if cs['raw_k_pre'] is not None:
                cs['raw_k_pre'].copy_(cf['raw_k_pre'])


def check(name, cfg, device, history, tails, steps):
    weights = RandomWeights(cfg, device, seed=0)
    full = LatentDecodeRuntime(cfg, weights, history, tails, device, extra_windows=1)
    split = LatentDecodeRuntime(cfg, weights, history, tails, device, extra_windows=1, seq_split=True)
    copy_shard(full, split)
    tokens = torch.randint(0, cfg.vocab, (len(history),), generator=torch.Generator().manual_seed(7)).to(device)
    worst = 0.0

    def compare(a, b):
        nonlocal worst
        err = (a.float() - b.float()).abs().max().item()
        worst = max(worst, err)
        assert err <= 2e-2, f'{name}: logits differ by {err}'

    for _ in range(steps):
        full.tokens.copy_(tokens)
        split.tokens.copy_(tokens)
        compare(full.step_eager(), split.step_eager())
        tokens = full.next_tokens().clone()
    for rt in (full, split):
        rt.tokens.copy_(tokens)
        rt.capture(warmup=1)
    for _ in range(3):
        compare(full.step(), split.step())
        tokens = full.next_tokens().clone()
        full.tokens.copy_(tokens)
        split.tokens.copy_(tokens)
    torch.cuda.synchronize()
    full.graph = split.graph = None            # graphs holding NCCL calls go before the process group
    return worst


def main():
    dist.init_process_group('nccl', timeout=timedelta(seconds=120))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    results = {}
    # Llama-3.1-8B r4 (the tcgen05 latent route); tails near the window end
    # so that Beacons are inserted and a window completes during the steps.
    results['llama'] = check('llama', LatentLlamaConfig(layers=2), device, [2048, 1536, 768], [1015, 7, 500], 12)
    # Qwen2.5-14B r2 geometry (40 heads, rank 512: the split-KV route, biases).
    results['qwen'] = check('qwen', dataclasses.replace(qwen25_14b_r2(), layers=2), device, [3072, 256],
                            [1021, 300], 8)
    gc.collect()
    torch.cuda.synchronize()
    dist.barrier()
    if dist.get_rank() == 0:
        print('PASS', results, flush=True)
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
