"""The reconstruct decode backend (oracle, test-only).

Restates ``reconstruction_attention`` (tools/benchmark/context_decode_runtime.py
:298-344) on top of ``ReconstructionCache.materialize`` (slimkv/llama3/memory.py
:26-48): every Beacon key and value is rebuilt from its latent by the bf16
up-projection ``nn.Linear`` (one rounding of the fp32-accumulated product plus
bias), queries and raw keys are rotated (BF16-exact RoPE), Beacon keys are not,
and one grouped attention runs over all keys; with a Beacon inserted this step
(``size``) it is the last key and the raw token's query does not see it
(bottom-right causal, context_decode_runtime.py:337-339).
"""
import math

import numpy as np

from .attention import eager_attention
from .bf16 import round_bf16
from .rope import rope_bf16


def materialize(latent, weight, bias=None):
    """``bf16(latent @ weight.T + bias)`` for latents ``[..., R]`` and an
    ``nn.Linear`` weight ``[Hkv*D, R]`` (memory.py:31-38)."""
    full = np.asarray(latent, np.float64) @ np.asarray(weight, np.float64).T
    if bias is not None:
        full = full + np.asarray(bias, np.float64)
    return round_bf16(full)


def reconstruct_decode_attention(q, raw_k, raw_v, latent_k, latent_v, uk, uv, cos, sin, query_positions,
                                 raw_positions, size, uk_bias=None, uv_bias=None):
    """One sequence (``B = 1``) of the reconstruct backend before ``o_proj``.

    ``q [1, L, H, d]`` pre-RoPE (``L = 1 + size``), ``raw_k / raw_v [1, S, Hkv,
    d]`` pre-RoPE raw keys and values (sinks, tail, current token) rotated at
    ``raw_positions [1, S]``, ``latent_k / latent_v [1, N, R]`` (with this step's
    Beacon last when ``size``).  Returns float64 ``out [1, L, H*d]`` and the
    reconstructed ``key / value [1, N, Hkv, d]`` (bf16 values).
    """
    batch, length, heads, dim = q.shape
    kv_heads = raw_k.shape[2]
    q_rot = rope_bf16(q, cos, sin, np.asarray(query_positions)[:, :, None])
    k_rot = rope_bf16(raw_k, cos, sin, np.asarray(raw_positions)[:, :, None])
    n = latent_k.shape[1]
    key = materialize(latent_k, uk, uk_bias).reshape(batch, n, kv_heads, dim)
    value = materialize(latent_v, uv, uv_bias).reshape(batch, n, kv_heads, dim)
    k_all = np.concatenate([k_rot, key], axis=1)
    v_all = np.concatenate([np.asarray(raw_v, np.float64), value], axis=1)
    out, _ = eager_attention(q_rot, k_all, v_all, 1.0 / math.sqrt(dim), bool(size))
    return {'out': out.reshape(batch, length, heads * dim), 'key': key, 'value': value, 'q_rot': q_rot,
            'k_rot': k_rot}
