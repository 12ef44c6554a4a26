"""Split-count heuristics of the reference decode extension (oracle, test-only)."""
import math


def latent_splits(key_length, grid_heads, sm_count):
    """Width-320 split count (kernels/fa2_decode/binding.cpp:94-105).

    ``blocks = ceil(N / 64)``; ``splits = min(32, blocks, ceil(SMs /
    grid_heads))``, then reduced while one fewer split still covers every
    block with the same per-split block count.
    """
    blocks = (key_length + 63) // 64
    splits = min(32, blocks, (sm_count + grid_heads - 1) // grid_heads)
    while splits > 1 and (splits - 1) * ((blocks + splits - 1) // splits) >= blocks:
        splits -= 1
    return splits


def dense_splits(grid, sms, blocks):
    """FA2 occupancy heuristic (kernels/fa2_decode/binding.cpp:17-33)."""
    if grid >= 0.8 * sms:
        return 1
    limit = min(128, sms, blocks)
    eff = {}
    for s in range(1, limit + 1):
        if s > 1 and math.ceil(blocks / s) == math.ceil(blocks / (s - 1)):
            continue
        waves = grid * s / sms
        eff[s] = waves / math.ceil(waves)
    best = max(eff.values())
    for s in range(1, limit + 1):
        if eff.get(s, 0.0) >= 0.85 * best:
            return s
    return 1


def original_splits(width, key_length, query_heads, sm_count):
    """Split count of an unpacked Q2 launch (slimkv/llama3/paired_decode.py:5-27)."""
    if width == 320:
        return latent_splits(key_length, query_heads, sm_count)
    block_n = 128 if width <= 128 else 64
    return dense_splits(query_heads, 2 * sm_count, (key_length + block_n - 1) // block_n)
