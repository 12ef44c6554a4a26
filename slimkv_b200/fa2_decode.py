"""Drop-in for the reference's latent decode step ``slimkv.llama3.fa2_decode``.

``decode(attention, hidden, position_ids, past_key_value, forward=None)`` keeps
the contract of the reference's ``decode`` (slimkv/llama3/fa2_decode.py:77-166):
the same arguments, the same return value ``(o_proj output, None,
ReconstructionCacheUpdate)`` and the same errors, so the reference's attention
modules can call it in place of their own (``LlamaAttention.forward``,
modeling_llama.py:1403-1404; ``LlamaFlashAttention2.forward``, 1648-1649).

What runs where:

* the projections stay the module's own ``nn.Linear`` layers (cuBLAS):
  ``q_proj``, ``k_proj``/``v_proj`` of the raw token and, on a Beacon-insertion
  step, ``beacon_q_proj`` and the K/V down-projections of the Beacon
  (fa2_decode.py:89-99);
* steps 3-8 — RoPE of the queries, raw-branch grouped attention, q-absorb into
  Beacon-K latent space, latent split-KV attention (causal on an insertion
  step), V up-projection with its bias, K-bias LSE shift and the LSE merge —
  are one call of the fused sm_100a decode (``slimkv_latent_decode``), whose
  latent branch for 32 query heads and ranks up to 320 is the tcgen05 kernel;
* the reference's cache is kept as it is: its ``ReconstructionCache`` holds
  pre-RoPE sink and raw keys and separate history / window latent tensors, so
  each call rotates the raw keys at their compressed positions
  (``slimkv_rope_decode``, the BF16-exact rule of decode_kernels.py:8-51) and
  gathers them and the latents into the fused op's token-major buffers — the
  same O(N) assembly the reference performs with ``cat_tensor``
  (fa2_decode.py:103-106).  The native runtime (``slimkv_b200.runtime``) keeps
  its caches in that layout and skips this step.

There is no CPU path: CPU tensors, dtypes other than bf16 and geometries the
fused op does not support raise.  ``forward`` selects the attention
implementation in the reference (FA2 or eager); here the fused kernel is the
implementation, so only ``forward=None`` is accepted.
"""
import math

import torch

from . import kernels

_ROPE_TYPES = ('RotaryEmbedding', 'LinearScalingRotaryEmbedding', 'Llama3RotaryEmbedding')


def _update_class():
    """The reference's ``ReconstructionCacheUpdate`` when the reference is
    importable (its ``LlamaMemory.update_memory`` checks the type), else the
    structural mirror below."""
    try:
        from slimkv.llama3.memory import ReconstructionCacheUpdate as ref
        return ref
    except Exception:
        return ReconstructionCacheUpdate


class ReconstructionCacheUpdate(tuple):
    """Mirror of the reference's four-item cache update
    (slimkv/llama3/memory.py:51-58): ``(key, value, beacon_size,
    beacon_indices)`` with the new Beacon latents as attributes."""

    def __new__(cls, key, value, beacon_size, beacon_indices, key_latents, value_latents):
        result = super().__new__(cls, (key, value, beacon_size, beacon_indices))
        result.key_latents = key_latents
        result.value_latents = value_latents
        return result


def _uses_latent_decode(config):
    return getattr(config, 'beacon_decode_backend', 'reconstruct') in ('latent', 'fa2')


def eligible(attention, hidden_states, past_key_value, output_attentions):
    """The reference's eligibility test (fa2_decode.py:69-74), with the
    cache type checked by its fields so that the reference's
    ``ReconstructionCache`` and structural stand-ins both qualify."""
    cache = past_key_value[0] if past_key_value is not None else None
    return (getattr(attention.config, '_slimkv_decode_step', False)
            and _uses_latent_decode(attention.config)
            and all(hasattr(cache, f) for f in ('sink', 'history', 'raw', 'window', 'window_raw_indices'))
            and not attention.training and not output_attentions
            and hidden_states.shape[0] > 0 and hidden_states.shape[1] in (1, 2))


def _len(t):
    return 0 if t is None else t.shape[2]


def _project(attention, hidden, size):
    """Projections of fa2_decode.py:88-99."""
    batch = hidden.shape[0]
    raw_hidden = hidden[:, :1]
    q = attention.q_proj(hidden)
    new_k = attention.k_proj(raw_hidden).reshape(batch, 1, attention.num_key_value_heads,
                                                attention.head_dim).transpose(1, 2)
    new_v = attention.v_proj(raw_hidden).reshape_as(new_k.transpose(1, 2)).transpose(1, 2)
    kl = vl = None
    if size:
        if 'q' in attention.config.beacon_param:
            q = torch.cat([q[:, :1], attention.beacon_q_proj(hidden[:, 1:])], dim=1)
        shared = getattr(attention, '_use_shared_kv_down_proj', lambda: False)()
        kd = attention.beacon_kv_down_proj if shared else attention.beacon_k_down_proj
        vd = attention.beacon_kv_down_proj if shared else attention.beacon_v_down_proj
        kl, vl = kd(hidden[:, 1:]).unsqueeze(1), vd(hidden[:, 1:]).unsqueeze(1)
    return q, new_k, new_v, kl, vl


def decode_attention(attention, hidden, position_ids, past_key_value, out_dtype=None):
    """Steps 1-8 of ``decode`` without ``o_proj``: returns ``(attn [B, L, H*D],
    update)``.  ``out_dtype`` torch.float32 gives the fp32-accumulated result
    before any bf16 rounding (the fused op's fp32 output mode)."""
    pk, pv, size, indices = past_key_value
    batch, length, _ = hidden.shape
    if size not in (0, 1) or length != size + 1:
        raise ValueError('Latent decode expects one raw token followed by at most one Beacon.')
    uk, uv = attention.beacon_k_up_proj, attention.beacon_v_up_proj
    if not isinstance(uk, torch.nn.Linear) or not isinstance(uv, torch.nn.Linear):
        raise ValueError('Latent decode currently requires globally coupled Linear up projections.')
    if not hidden.is_cuda or hidden.dtype != torch.bfloat16:
        raise ValueError('slimkv_b200 decode runs bf16 models on CUDA devices')
    heads, kv_heads, dim = attention.num_heads, attention.num_key_value_heads, attention.head_dim
    rope = attention.rotary_emb
    if type(rope).__name__ not in _ROPE_TYPES or position_ids.shape[-1] > rope.max_seq_len_cached:
        raise ValueError('slimkv_b200 decode needs a table-based rotary embedding covering the positions')
    device = hidden.device
    update_cls = _update_class()

    q, new_k, new_v, kl, vl = _project(attention, hidden, size)
    update = update_cls(new_k, new_v, size, indices, kl, vl)
    update.raw_only = True

    # Raw keys: sinks, the open window's raw tail and this step's token, rotated
    # at their compressed positions (fa2_decode.py:109-145) into the fused
    # op's token-major cache [B, K, Hkv, D].
    sink_len, history_len = _len(pk.sink), _len(pk.history)
    parts_k = [t for t in (pk.sink, pk.raw, new_k) if t is not None]
    parts_v = [t for t in (pv.sink, pv.raw, new_v) if t is not None]
    raw_k = torch.cat(parts_k, dim=2) if len(parts_k) > 1 else new_k
    raw_v = torch.cat(parts_v, dim=2) if len(parts_v) > 1 else new_v
    keys = raw_k.shape[2]
    qpos = position_ids[:, -length:].to(torch.int64).contiguous()
    q4 = q.reshape(batch, length, heads, dim)
    cos = rope.cos_cached.to(device=device, dtype=torch.float32).contiguous()
    sin = rope.sin_cached.to(device=device, dtype=torch.float32).contiguous()
    _, k_rot = kernels.rope_decode(q4.transpose(1, 2), raw_k, cos, sin, qpos, pk.window_raw_indices,
                                   sink_len, history_len)
    cap = (keys + 63) // 64 * 64
    raw_k_rot = torch.empty(batch, cap, kv_heads, dim, dtype=torch.bfloat16, device=device)
    raw_vt = torch.empty_like(raw_k_rot)
    raw_k_rot[:, :keys].copy_(k_rot.transpose(1, 2))
    raw_vt[:, :keys].copy_(raw_v.transpose(1, 2))

    # Latents: history, open-window Beacons and this step's Beacon, one row
    # [K latent | V latent] per Beacon (fa2_decode.py:105-106).
    rank_k, rank_v = uk.in_features, uv.in_features
    lat_parts = [(a, b) for a, b in ((pk.history, pv.history), (pk.window, pv.window), (kl, vl)) if a is not None]
    n_lat = sum(a.shape[2] for a, _ in lat_parts)
    lcap = max(64, (n_lat + 63) // 64 * 64)
    lat = torch.empty(batch, lcap, rank_k + rank_v, dtype=torch.bfloat16, device=device)
    at = 0
    for a, b in lat_parts:
        n = a.shape[2]
        lat[:, at:at + n, :rank_k].copy_(a[:, 0])
        lat[:, at:at + n, rank_k:].copy_(b[:, 0])
        at += n

    i32 = dict(dtype=torch.int32, device=device)
    out = torch.empty(batch, length, heads * dim, dtype=out_dtype or torch.bfloat16, device=device)
    kernels.latent_decode(
        q=q4, raw_k_rot=raw_k_rot, raw_v=raw_vt, lat_k=lat[..., :rank_k], lat_v=lat[..., rank_k:],
        raw_len=torch.full((batch,), keys, **i32), latent_len=torch.full((batch,), n_lat, **i32),
        qpos=qpos.to(torch.int32), uk=uk.weight, uv=uv.weight, uk_bias=uk.bias, uv_bias=uv.bias,
        cos=cos, sin=sin, out=out, scale=1.0 / math.sqrt(dim),
        latent_len_max=n_lat, raw_len_max=keys)
    return out, update


def decode(attention, hidden, position_ids, past_key_value, forward=None):
    """One raw token, optionally followed by its newly inserted Beacon.

    The reference's ``decode`` (slimkv/llama3/fa2_decode.py:77-166) with steps
    3-8 in the fused sm_100a decode.  Returns ``(attention.o_proj_with_beacon
    (output, size, indices), None, update)`` where ``update`` carries the new
    raw K/V and Beacon latents for ``LlamaMemory.update_memory``."""
    if forward is not None:
        raise ValueError('slimkv_b200 decode computes attention with its fused kernel; pass forward=None')
    output, update = decode_attention(attention, hidden, position_ids, past_key_value)
    _, size, indices = past_key_value[1:]
    return attention.o_proj_with_beacon(output, size, indices), None, update
