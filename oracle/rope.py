"""BF16-exact rotary embedding (oracle, test-only)."""
import math

import numpy as np

from .bf16 import round_bf16


def rope_tables(head_dim, base, max_positions, scaling=None):
    """fp32 cos/sin tables ``[max_positions, head_dim]``.

    Restates ``RotaryEmbedding`` and ``Llama3RotaryEmbedding`` table
    construction (slimkv/modeling_utils.py:354-372 and 690-735).  The
    reference builds these tables on the CPU in fp32 with torch
    (slimkv/vllm_plugin/model.py:69-79 insists on CPU construction because
    GPU pow/sin/cos round differently), so the oracle uses CPU torch for the
    same fp32 operations.  ``scaling`` is ``None`` or a dict with ``factor``,
    ``original_max_position_embeddings``, ``low_freq_factor``,
    ``high_freq_factor`` (Llama-3 scaling).
    """
    import torch
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    if scaling is not None:
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
        inv = torch.tensor(adjusted, dtype=torch.float32)
    t = torch.arange(max_positions, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().numpy(), emb.sin().numpy()


def rope_bf16(x, cos, sin, positions):
    """Rotate bf16 values ``x [..., D]`` at integer ``positions [...]``.

    Restates the decode rotary (slimkv/llama3/fa2_decode.py:116-119 and the
    fused kernel slimkv/llama3/decode_kernels.py:8-51): with
    ``c = bf16(cos[p])`` and ``s = bf16(sin[p])`` every product is rounded to
    bf16 and so is the sum, ``out = bf16(bf16(x*c) + bf16(rotate_half(x)*s))``
    where ``rotate_half(x) = cat(-x[D/2:], x[:D/2])``.
    ``x`` must already hold bf16 values (as fp32).  Returns fp32 holding bf16.
    """
    x = np.asarray(x, dtype=np.float32)
    pos = np.asarray(positions)
    half = x.shape[-1] // 2
    c = round_bf16(np.asarray(cos, np.float32)[pos])
    s = round_bf16(np.asarray(sin, np.float32)[pos])
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    first = round_bf16(x * c)
    second = round_bf16(rot * s)
    return round_bf16(first + second)


def raw_key_positions(sink, window_raw_indices, history, current):
    """Compressed positions of the raw-branch keys of one decode step.

    Restates fa2_decode.py:127-131: sinks sit at ``0..sink-1``, the raw tail
    token ``i`` of the current window at ``window_raw_indices[i] + sink +
    history`` and the current raw token at ``current`` (the first query
    position of the step).
    """
    parts = [np.arange(sink, dtype=np.int64)]
    if window_raw_indices is not None and len(window_raw_indices):
        parts.append(np.asarray(window_raw_indices, np.int64) + sink + history)
    parts.append(np.array([current], dtype=np.int64))
    return np.concatenate(parts)
