"""CPU restatement of a prefill chunk's attention over a latent history (test
infrastructure: the checker of ``slimkv_b200.prefill_attention``).

The reference materialises the Beacon keys and values of every history
latent through the up-projections (``ReconstructionCache.materialize``,
slimkv/llama3/memory.py:26-48: ``up(latent)`` reshaped to [Hkv, D] per
token, ``cat_tensor([sink, history, recent, current])``) and runs one causal
flash attention over the joined keys with the chunk's rows as the last
queries (modeling_llama.py:1650-1681 and ``_flash_attention_forward``):
query token t of a chunk of T tokens sees every key before the chunk and the
chunk's keys up to its own.  Beacon keys carry no rotary, so the history
keys are the plain up-projections.  Here in float64 numpy.
"""
import numpy as np

from .bf16 import round_bf16


def materialize(lat, up, bias, kv_heads, head_dim, bf16_out=False):
    """up(latent) [N, R] -> [N, Hkv, D] (nn.Linear: lat @ up.T + bias);
    ``bf16_out`` rounds the result as the reference's bf16 Linear does."""
    full = np.asarray(lat, np.float64) @ np.asarray(up, np.float64).T
    if bias is not None:
        full = full + np.asarray(bias, np.float64)
    if bf16_out:
        full = round_bf16(full.astype(np.float32)).astype(np.float64)
    return full.reshape(len(lat), kv_heads, head_dim)


def prefill_attention(q, prefix_k, prefix_v, lat_k, lat_v, uk, uv, k_cur, v_cur, scale, uk_bias=None,
                      uv_bias=None, bf16_history=False):
    """One sequence.  q [T, H, D] (rotated chunk queries), prefix_k/v [P, Hkv,
    D] (sinks and any raw keys before the chunk), lat_k/v [N, R] (history
    latents), uk/uv [Hkv*D, R], k_cur/v_cur [T, Hkv, D] (the chunk's keys,
    rotated where the reference rotates them).  Returns (out [T, H, D], lse
    [T, H]) in float64.  ``bf16_history`` rounds the materialised history
    keys and values to bf16 (the reference's bf16 modules)."""
    T, H, D = q.shape
    Hkv = k_cur.shape[1]
    group = H // Hkv
    hk = materialize(lat_k, uk, uk_bias, Hkv, D, bf16_history)
    hv = materialize(lat_v, uv, uv_bias, Hkv, D, bf16_history)
    keys = np.concatenate([np.asarray(prefix_k, np.float64), hk, np.asarray(k_cur, np.float64)])
    vals = np.concatenate([np.asarray(prefix_v, np.float64), hv, np.asarray(v_cur, np.float64)])
    before = len(prefix_k) + len(lat_k)
    out = np.zeros((T, H, D))
    lse = np.zeros((T, H))
    qf = np.asarray(q, np.float64)
    for h in range(H):
        g = h // group
        s = (qf[:, h] @ keys[:, g].T) * scale                       # [T, keys]
        visible = np.arange(len(keys))[None, :] <= before + np.arange(T)[:, None]
        s = np.where(visible, s, -np.inf)
        m = s.max(-1, keepdims=True)
        p = np.exp(s - m)
        tot = p.sum(-1, keepdims=True)
        out[:, h] = (p @ vals[:, g]) / tot
        lse[:, h] = (m + np.log(tot))[:, 0]
    return out, lse
