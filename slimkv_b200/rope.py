"""Rotary tables built exactly like the reference.

The reference builds its cos/sin caches on the CPU in fp32 with torch
(``RotaryEmbedding`` / ``Llama3RotaryEmbedding``,
slimkv/modeling_utils.py:354-372 and 690-735) and its vLLM adapter insists on
CPU construction because GPU pow/sin/cos round differently
(slimkv/vllm_plugin/model.py:69-79).  BF16-exact RoPE needs bit-identical
tables, so these are built the same way and then copied to the device.
"""
import math

import torch

LLAMA3_SCALING = dict(factor=8.0, original_max_position_embeddings=8192, low_freq_factor=1.0,
                      high_freq_factor=4.0)


def inverse_frequencies(head_dim, base, scaling=None):
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    if scaling is None:
        return inv
    factor = scaling['factor']
    original = scaling.get('original_max_position_embeddings', 8192)
    low = scaling.get('low_freq_factor', 1)
    high = scaling.get('high_freq_factor', 4)
    low_wavelen, high_wavelen = original / low, original / high
    adjusted = []
    for freq in inv:
        wavelen = 2 * math.pi / freq
        if wavelen < high_wavelen:
            adjusted.append(freq)
        elif wavelen > low_wavelen:
            adjusted.append(freq / factor)
        else:
            smooth = (original / wavelen - low) / (high - low)
            adjusted.append((1 - smooth) * freq / factor + smooth * freq)
    return torch.tensor(adjusted, dtype=torch.float32)


def rope_tables(head_dim, base, positions, scaling=None, device=None):
    """Return fp32 ``(cos, sin)`` tables ``[positions, head_dim]`` on ``device``."""
    with torch.device('cpu'):
        inv = inverse_frequencies(head_dim, base, scaling)
        t = torch.arange(positions, dtype=torch.float32)
        emb = torch.cat([torch.outer(t, inv)] * 2, dim=-1)
        cos, sin = emb.cos(), emb.sin()
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin
