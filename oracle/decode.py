"""One decode step of SlimKV latent attention (oracle, test-only)."""
import math

import numpy as np

from .attention import eager_attention, merge_attention, project_query, project_value
from .bf16 import round_bf16
from .rope import rope_bf16


def rope_fp32(x, cos, sin, positions):
    """fp32 rotary with fp32 rounding per operation (fp32 models)."""
    x = np.asarray(x, np.float32)
    pos = np.asarray(positions)
    half = x.shape[-1] // 2
    c = np.asarray(cos, np.float32)[pos]
    s = np.asarray(sin, np.float32)[pos]
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * c).astype(np.float32) + (rot * s).astype(np.float32)


def latent_decode_attention(q, raw_k, raw_v, latent_k, latent_v, uk, uv, cos, sin,
                            query_positions, raw_positions, size, uk_bias=None,
                            uv_bias=None, dtype='bf16', lengths=None, raw_lengths=None):
    """Attention of one decode step over the compressed cache, before ``o_proj``.

    Restates steps 3-8 of ``decode`` (slimkv/llama3/fa2_decode.py:77-166)
    with the eager backend (slimkv/llama3/latent_decode.py:16-41):

    * ``q [B, L, H, d]`` pre-RoPE queries (raw token, then the Beacon on an
      insertion step, ``L = 1 + size``); rotated at ``query_positions [B, L]``.
    * ``raw_k/raw_v [B, S, Hkv, d]`` pre-RoPE sink + raw tail + current raw
      token; keys rotated at ``raw_positions [B, S]`` (fa2_decode.py:122-132).
    * ``latent_k [B, N, R_k]``, ``latent_v [B, N, R_v]``: history + window +
      new Beacon latents (one shared latent "head"; Beacon K has no RoPE).
    * ``uk``/``uv``: up-projection weights ``[Hkv*d, R]``.
    * raw branch: non-causal grouped attention (fa2_decode.py:146-148);
      latent branch: q-absorb, causal only when ``size`` (bottom-right),
      V up-projection (152-156); ``uk_bias`` shifts the latent LSE by
      ``scale * q . b_k[g]`` and ``uv_bias`` is added to the up-projected
      output (157-163); then the LSE merge (164).
    ``lengths`` / ``raw_lengths`` optionally give per-row key counts.

    Returns a dict of float64 arrays: ``q_rot`` (BLHd), ``raw_out`` (BHLd),
    ``raw_lse``, ``q_lat`` (BHLR), ``latent_branch_out`` (BLHR) and
    ``latent_branch_lse`` (before the bias shift), ``latent_lse``,
    ``latent_out`` (BHLd after up-projection and bias) and ``out``
    (``[B, L, H*d]``).
    """
    batch, length, heads, dim = q.shape
    kv_heads = raw_k.shape[2]
    rotate = rope_bf16 if dtype == 'bf16' else rope_fp32
    q_rot = rotate(q, cos, sin, np.asarray(query_positions)[:, :, None])
    k_rot = rotate(raw_k, cos, sin, np.asarray(raw_positions)[:, :, None])
    scale = 1.0 / math.sqrt(dim)
    raw_out, raw_lse = eager_attention(q_rot, k_rot, raw_v, scale, False, raw_lengths)
    raw_out = raw_out.transpose(0, 2, 1, 3)                        # BHLd
    result = {'q_rot': q_rot, 'k_rot': k_rot, 'raw_out': raw_out, 'raw_lse': raw_lse}
    if latent_k is None or latent_k.shape[1] == 0:
        merged = raw_out
    else:
        q_lat = project_query(q_rot.transpose(0, 2, 1, 3), uk, kv_heads)  # BHLR
        lat_out, lat_lse = eager_attention(q_lat.transpose(0, 2, 1, 3), latent_k[:, :, None],
                                           latent_v[:, :, None], scale, bool(size), lengths)
        result.update(latent_branch_out=lat_out, latent_branch_lse=lat_lse)
        lat_out = project_value(lat_out.transpose(0, 2, 1, 3), uv, kv_heads)  # BHLd
        if uk_bias is not None:
            group = heads // kv_heads
            bias = np.repeat(np.asarray(uk_bias, np.float64).reshape(kv_heads, dim), group, axis=0)
            lat_lse = lat_lse + (q_rot.transpose(0, 2, 1, 3) * bias[None, :, None]).sum(-1) * scale
        if uv_bias is not None:
            group = heads // kv_heads
            bias = np.repeat(np.asarray(uv_bias, np.float64).reshape(kv_heads, dim), group, axis=0)
            lat_out = lat_out + bias[None, :, None]
        merged = merge_attention(raw_out, raw_lse, lat_out, lat_lse)
        result.update(q_lat=q_lat, latent_lse=lat_lse, latent_out=lat_out)
    result['out'] = merged.transpose(0, 2, 1, 3).reshape(batch, length, heads * dim)
    return result


__all__ = ['latent_decode_attention', 'rope_fp32', 'round_bf16']
