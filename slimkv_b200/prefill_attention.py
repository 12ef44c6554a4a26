"""Prefill attention of a chunk whose history is kept as Beacon latents.

The reference joins every prefill chunk's attention by materialising the
Beacon keys and values of all history latents through the up-projections
(``ReconstructionCache.materialize``, slimkv/llama3/memory.py:26-48, joined
in the prefill forward at modeling_llama.py:1650-1681) and running one causal
flash attention over [sinks, history, chunk]; that up-projection of the whole
history is repeated for every window of the prompt.  Beacon keys carry no
rotary, so here the history part runs in latent space instead:

1. queries absorbed into the latent key space per KV head (``q . U_k[g]``,
   bf16 like the reference's materialised keys);
2. ``slimkv_prefill_attention`` over the history latents, every head of the
   chunk a row of the one latent head (tcgen05 flash attention, width = the
   latent rank), with the K up-projection bias as a per-row LSE shift;
3. the latent output up-projected once per row (``U_v[g]``, + V bias);
4. ``slimkv_prefill_attention`` over the sinks (and any raw keys before the
   chunk) and the chunk's own keys, causal with bottom-right alignment;
5. the two parts merged by their LSEs (``slimkv_merge``).

The absorbed history costs (R_k + R_v) / (2 D) times the attention FLOPs of
materialised keys (2.5x at rank 320) and saves the per-window up-projection
and its key / value buffers; ``materialized_history_attention`` runs the
other recipe (history materialised by ``slimkv_reconstruct_kv`` once, then
the same kernel in full dimension) for comparison.  There is no CPU path.
"""
import ctypes

import torch

from . import _lib
from .kernels import _require, _stream


def attention(q, k, v, kv_len, scale, rows_per_token, causal=False, causal_offset=0, out=None, lse=None,
              wait_limit_ns=0):
    """``slimkv_prefill_attention``: q ``[B, T, Hkv*R, dq]``, k ``[B, cap, Hkv,
    dq]``, v ``[B, cap, Hkv, dv]`` (bf16, last dim contiguous), kv_len int32
    ``[B]``.  Returns ``(out [B, T, Hkv*R, dv] bf16, lse [B, T, Hkv*R] fp32)``."""
    for t in (q, k, v):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 4 and t.stride(3) == 1,
                 'bf16 CUDA tensors [B, rows, heads, dim] with a contiguous last dimension')
    B, T, H, dq = q.shape
    kv_heads, dv = k.shape[2], v.shape[3]
    _require(k.shape[:3] == v.shape[:3] and k.shape[3] == dq and k.stride()[:3] == v.stride()[:3] and
             H == kv_heads * rows_per_token, 'k / v [B, cap, Hkv, d] with one stride set; H = Hkv * R')
    _require(kv_len.is_cuda and kv_len.dtype == torch.int32 and kv_len.numel() == B, 'int32 kv_len [B]')
    if out is None:
        out = torch.empty((B, T, H, dv), dtype=torch.bfloat16, device=q.device)
    if lse is None:
        lse = torch.empty((B, T, H), dtype=torch.float32, device=q.device)
    _require(out.shape == (B, T, H, dv) and out.stride(3) == 1 and lse.shape == (B, T, H) and lse.stride(2) == 1,
             'out [B, T, H, dv], lse [B, T, H]')
    a = _lib.PrefillAttentionArgs()
    a.batch, a.kv_heads, a.rows_per_token, a.tokens, a.dim_qk, a.dim_v = B, kv_heads, rows_per_token, T, dq, dv
    a.q, a.k, a.v, a.kv_len, a.out, a.lse = (q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_len.data_ptr(),
                                             out.data_ptr(), lse.data_ptr())
    a.q_stride[:] = list(q.stride()[:3])
    a.kv_stride[:] = list(k.stride()[:3])
    a.out_stride[:] = list(out.stride()[:3])
    a.lse_stride[:] = list(lse.stride()[:2])
    a.kv_capacity = k.shape[1]
    a.causal, a.causal_offset, a.scale = int(causal), int(causal_offset), float(scale)
    a.wait_limit_ns = int(wait_limit_ns)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().slimkv_prefill_attention(ctypes.byref(a), _stream()))
    return out, lse


def _merge(o_a, lse_a, o_b, lse_b):
    """LSE merge of two [B, T, H, D] parts (``slimkv_merge``) -> [B, T, H, D]."""
    from .kernels import merge
    bhtd = lambda t: t.permute(0, 2, 1, 3)
    lse_t = lambda t: t.permute(0, 2, 1)
    return merge(bhtd(o_b), lse_t(lse_b), bhtd(o_a), lse_t(lse_a)).permute(0, 2, 1, 3).contiguous()


def latent_history_attention(q, prefix_k, prefix_v, lat_k, lat_v, lat_len, uk, uv, k_cur, v_cur, scale,
                             uk_bias=None, uv_bias=None, prefix_len=None):
    """Attention of a prefill chunk over [prefix, latent history, chunk].

    q ``[B, T, H, D]`` (rotated queries of the chunk's rows), prefix_k / v
    ``[B, P, Hkv, D]`` (sinks and raw keys before the chunk; ``prefix_len``
    int32 ``[B]`` of them valid, default all), lat_k / lat_v ``[B, cap, R]``
    (history latents, ``lat_len`` int32 ``[B]`` valid), uk / uv ``[Hkv*D, R]``
    (nn.Linear weights of the up-projections, biases ``[Hkv*D]`` or None),
    k_cur / v_cur ``[B, T, Hkv, D]`` (the chunk's keys as the reference
    attends them).  Every row of the chunk sees all prefix and history keys
    and the chunk's keys up to its own.  Returns ``[B, T, H, D]`` bf16.
    """
    B, T, H, D = q.shape
    kv_heads = k_cur.shape[2]
    group = H // kv_heads
    P = prefix_k.shape[1]
    rk, rv = lat_k.shape[-1], lat_v.shape[-1]
    dev = q.device
    # 1. absorb: q_lat[b, t, h] = q[b, t, h] . U_k[g(h)]  (U_k[g] = uk[g*D:(g+1)*D] : [D, R]), one GEMM
    #    per KV head over all the chunk's rows of its group.
    q5 = q.view(B, T, kv_heads, group, D)
    q_lat = torch.einsum('btgjd,gdr->btgjr', q5, uk.view(kv_heads, D, rk)).reshape(B, T, H, rk)
    # 2. history in latent space: all H heads are rows of the one latent head.
    o_lat, lse_h = attention(q_lat, lat_k.unsqueeze(2), lat_v.unsqueeze(2), lat_len, scale, H)
    if uk_bias is not None:
        # every history key carries the bias: its score adds q . b_k[g], a row constant
        shift = torch.einsum('btgjd,gd->btgj', q5.float(), uk_bias.float().view(kv_heads, D)).reshape(B, T, H)
        lse_h = lse_h + shift * scale
    # 3. up-project the latent output: o[b, t, h] = o_lat[b, t, h] . U_v[g]^T (+ b_v)
    o_hist = torch.einsum('btgjr,gdr->btgjd', o_lat.view(B, T, kv_heads, group, rv),
                          uv.view(kv_heads, D, rv)).reshape(B, T, H, D)
    if uv_bias is not None:
        o_hist = o_hist + uv_bias.view(kv_heads, 1, D).expand(kv_heads, group, D).reshape(H, D)
    # 4. prefix + chunk, causal bottom-right (the chunk's rows are the last P + T keys' queries)
    keys_k = torch.cat([prefix_k, k_cur], dim=1)
    keys_v = torch.cat([prefix_v, v_cur], dim=1)
    if prefix_len is None:
        kv_len = torch.full((B,), P + T, dtype=torch.int32, device=dev)
    else:
        _require(bool((prefix_len == P).all()), 'ragged prefixes are not supported: pad the prefix to P')
        kv_len = prefix_len + T
    o_cur, lse_c = attention(q, keys_k, keys_v, kv_len, scale, group, causal=True, causal_offset=P)
    # 5. merge the parts by their LSEs
    return _merge(o_hist, lse_h, o_cur, lse_c)


def materialized_history_attention(q, prefix_k, prefix_v, lat_k, lat_v, n_hist, uk, uv, k_cur, v_cur, scale,
                                   uk_bias=None, uv_bias=None):
    """The same attention with the history materialised, as the reference does
    (``slimkv_reconstruct_kv`` writes the bf16 Beacon keys / values of the
    first ``n_hist`` latents of every sequence between the prefix and the
    chunk), then one causal ``slimkv_prefill_attention`` in full dimension.
    Arguments as ``latent_history_attention`` with one history length for the
    batch.  Returns ``[B, T, H, D]`` bf16."""
    from .reconstruct import reconstruct_kv
    B, T, H, D = q.shape
    kv_heads = k_cur.shape[2]
    P = prefix_k.shape[1]
    n_hist = int(n_hist)
    keys = torch.empty((B, P + n_hist + T, kv_heads, D), dtype=torch.bfloat16, device=q.device)
    vals = torch.empty_like(keys)
    keys[:, :P] = prefix_k
    vals[:, :P] = prefix_v
    keys[:, P + n_hist:] = k_cur
    vals[:, P + n_hist:] = v_cur
    if n_hist:
        start = torch.full((B,), P, dtype=torch.int32, device=q.device)
        reconstruct_kv(lat_k, lat_v, uk, uv, keys, vals, n_hist, b_k_up=uk_bias, b_v_up=uv_bias, out_start=start)
    kv_len = torch.full((B,), P + n_hist + T, dtype=torch.int32, device=q.device)
    out, _ = attention(q, keys, vals, kv_len, scale, H // kv_heads, causal=True, causal_offset=P + n_hist)
    return out
