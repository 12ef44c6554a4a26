"""Eager attention, LSE merge and the latent projections (oracle, test-only).

All arithmetic is float64 so the oracle is at least as exact as the
reference's fp32 eager path.
"""
import numpy as np


def eager_attention(q, k, v, scale, causal=False, lengths=None):
    """Grouped attention over one decode step, returning ``(out, lse)``.

    Restates ``eager_forward`` (slimkv/llama3/latent_decode.py:16-41):
    BSHD inputs ``q [B, Q, H, Dk]``, ``k [B, N, Hkv, Dk]``, ``v [B, N, Hkv, Dv]``
    with ``H % Hkv == 0``; query head ``h`` reads KV head ``h // (H // Hkv)``.
    ``causal`` is bottom-right aligned: query ``i`` sees keys ``j`` with
    ``j <= i + N - Q`` (latent_decode.py:30-33).  A row that sees no key gets
    zero output and ``lse = -inf`` (latent_decode.py:36-37).
    ``lengths`` (optional, per batch row) truncates the keys of each row to
    its first ``lengths[b]`` entries, the ``cache_seqlens`` contract of the
    reference extension (kernels/fa2_decode/binding.cpp:83-90).
    Returns ``out [B, Q, H, Dv]`` (float64) and ``lse [B, H, Q]`` (float64).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    batch, queries, heads, _ = q.shape
    keys, kv_heads = k.shape[1], k.shape[2]
    if heads % kv_heads or k.shape[0] != batch or v.shape[:3] != k.shape[:3]:
        raise ValueError('invalid grouped attention shapes')
    group = heads // kv_heads
    out = np.zeros((batch, queries, heads, v.shape[-1]))
    lse = np.full((batch, heads, queries), -np.inf)
    for b in range(batch):
        n = keys if lengths is None else int(lengths[b])
        for h in range(heads):
            g = h // group
            kk, vv = k[b, :n, g], v[b, :n, g]
            s = q[b, :, h] @ kk.T * scale                     # [Q, n]
            if causal:
                qi = np.arange(queries)[:, None] + n - queries
                s = np.where(np.arange(n)[None, :] > qi, -np.inf, s)
            for i in range(queries):
                row = s[i]
                if n == 0 or not np.isfinite(row).any():
                    continue
                m = row.max()
                p = np.exp(row - m)
                total = p.sum()
                lse[b, h, i] = m + np.log(total)
                out[b, i, h] = (p / total) @ vv
    return out, lse


def merge_attention(raw_out, raw_lse, latent_out, latent_lse):
    """Softmax-mass merge of the raw and latent branches.

    Restates ``merge_attention`` (slimkv/llama3/fa2_decode.py:57-66) and its
    fused form (slimkv/llama3/decode_kernels.py:54-76):
    ``T = logaddexp(r, l)``, ``out = e^(r-T) raw + e^(l-T) latent``.
    Outputs are BHQD, LSE is BHQ.  A branch with ``lse = -inf`` contributes
    zero mass.
    """
    r = np.asarray(raw_lse, dtype=np.float64)
    l = np.asarray(latent_lse, dtype=np.float64)
    total = np.logaddexp(r, l)
    with np.errstate(invalid='ignore'):
        wr = np.where(np.isneginf(r), 0.0, np.exp(r - total))[..., None]
        wl = np.where(np.isneginf(l), 0.0, np.exp(l - total))[..., None]
    return wr * np.asarray(raw_out, np.float64) + wl * np.asarray(latent_out, np.float64)


def project_query(q, weight, kv_heads):
    """Absorb the query into Beacon-K latent space.

    Restates ``project_query`` (slimkv/llama3/fa2_decode.py:41-46):
    ``q [B, H, Q, d]`` and the up-projection weight ``U_k [Hkv*d, R]`` (an
    ``nn.Linear(R, Hkv*d)`` weight) give ``q_lat[b,h,i,:] = q[b,h,i,:] @
    U_k[g*d:(g+1)*d, :]`` with ``g = h // (H // Hkv)``.
    """
    q = np.asarray(q, np.float64)
    w = np.asarray(weight, np.float64)
    batch, heads, length, dim = q.shape
    group = heads // kv_heads
    w3 = w.reshape(kv_heads, dim, w.shape[-1])
    out = np.empty((batch, heads, length, w.shape[-1]))
    for h in range(heads):
        out[:, h] = q[:, h] @ w3[h // group]
    return out


def project_value(o, weight, kv_heads):
    """Up-project latent attention outputs to head dimension.

    Restates ``project_value`` (slimkv/llama3/fa2_decode.py:49-54):
    ``o [B, H, Q, R]`` with ``U_v [Hkv*d, R]`` gives
    ``out[b,h,i,:] = U_v[g*d:(g+1)*d, :] @ o[b,h,i,:]``.
    """
    o = np.asarray(o, np.float64)
    w = np.asarray(weight, np.float64)
    batch, heads, length, rank = o.shape
    dim = w.shape[0] // kv_heads
    group = heads // kv_heads
    w3 = w.reshape(kv_heads, dim, rank)
    out = np.empty((batch, heads, length, dim))
    for h in range(heads):
        out[:, h] = o[:, h] @ w3[h // group].T
    return out
