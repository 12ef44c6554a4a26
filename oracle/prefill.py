"""Prefill window compression and cache append (oracle, test-only).

Restates, on the CPU, what one interleaved prefill chunk does to a SlimKV
layer: the role-selected projections of ``qkv_proj_with_beacon``, the
Beacon-latent packing of ``_incremental_cache``, the prefill RoPE and the
cache writes of ``flush_memory``.  Role bookkeeping is integer work
(bit-exact); projections are fp64 products of bf16 values rounded once to
bf16, i.e. the correctly rounded result of the bf16 ``nn.Linear`` the
reference runs.
"""
import numpy as np

from .bf16 import round_bf16
from .pages import beacon_pages_append
from .rope import rope_bf16


def prefill_metadata(roles, chunk_rows):
    """``(raw_indices, beacon_indices, replicas)`` of the current chunk.

    Restates ``prepare_metadata`` (slimkv/llama3/prefill_ops.py:17-36): the
    chunk is the last ``chunk_rows`` entries of the window roles; raw rows
    have role 0, every other role is a Beacon row (role 2 marks a replica).
    """
    current = np.asarray(roles, np.int64)[-chunk_rows:] if chunk_rows else np.zeros(0, np.int64)
    return (np.nonzero(current == 0)[0], np.nonzero(current != 0)[0], bool((current == 2).any()))


def _linear(x, w, b=None, rnd=True):
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if b is not None:
        y = y + np.asarray(b, np.float64)
    y = y.astype(np.float32)
    return round_bf16(y) if rnd else y


def project_with_beacon(hidden, roles, weights, rnd=True, latents=None):
    """Role-selected q/k/v and Beacon latents of one chunk.

    Restates ``qkv_proj_with_beacon`` (slimkv/llama3/modeling_llama.py:
    1291-1345) with the low-rank Beacon projections
    ``_project_beacon_key/value`` (384-394, 446-456) and the latent packing
    of ``_incremental_cache`` (1347-1367) under prefill metadata:
    raw rows (role 0) take ``q_proj``/``k_proj``/``v_proj``; Beacon rows take
    ``beacon_q_proj``, latents ``h W_down^T`` and full keys/values
    ``up_proj(latent)`` (the latent rounded to bf16 first when ``rnd``, as a
    bf16 module does).  ``hidden [B, n, hidden]`` holds bf16 values;
    ``weights`` maps q, k, v, bq, k_down, v_down, k_up, v_up (nn.Linear
    weights [out, in]) and optional q_bias, k_bias, v_bias, bq_bias,
    k_up_bias, v_up_bias.  Returns a dict with ``query/key/value [B, n, .]``
    and ``key_latent/value_latent [B, n_beacon, R]`` (the rows of
    ``update.key_latents[:, 0]``), plus ``raw_indices`` / ``beacon_indices``.
    ``latents=(lk, lv)`` up-projects the given bf16 latents instead of the
    oracle's own (to check an up-projection on identical inputs).
    """
    hidden = np.asarray(hidden, np.float32)
    n = hidden.shape[1]
    raw, beacon, replicas = prefill_metadata(roles, n)
    if replicas:
        raise ValueError('replica Beacon rows need parallel windows (not on the prefill fast path)')
    w = weights
    hr, hb = hidden[:, raw], hidden[:, beacon]
    out = {'raw_indices': raw, 'beacon_indices': beacon}
    q = np.zeros(hidden.shape[:2] + (w['q'].shape[0],), np.float32)
    q[:, raw] = _linear(hr, w['q'], w.get('q_bias'), rnd)
    q[:, beacon] = _linear(hb, w['bq'], w.get('bq_bias'), rnd)
    lk = _linear(hb, w['k_down'], None, rnd)
    lv = _linear(hb, w['v_down'], None, rnd)
    kvd = w['k'].shape[0]
    k = np.zeros(hidden.shape[:2] + (kvd,), np.float32)
    v = np.zeros_like(k)
    k[:, raw] = _linear(hr, w['k'], w.get('k_bias'), rnd)
    v[:, raw] = _linear(hr, w['v'], w.get('v_bias'), rnd)
    uk, uv = (lk, lv) if latents is None else (np.asarray(latents[0], np.float32), np.asarray(latents[1], np.float32))
    k[:, beacon] = _linear(uk, w['k_up'], w.get('k_up_bias'), rnd)
    v[:, beacon] = _linear(uv, w['v_up'], w.get('v_up_bias'), rnd)
    out.update(query=q, key=k, value=v, key_latent=lk, value_latent=lv)
    return out


def prefill_rope(q, k, cos, sin, positions, roles, sink):
    """BF16-exact prefill rotary with Beacon keys left unrotated.

    Restates ``prefill_rope_kernel`` (slimkv/llama3/prefill_kernels.py:7-53)
    and the rule it fuses (``_apply_rotary_with_beacon``,
    slimkv/llama3/modeling_llama.py:1145-1178): ``q [B, Hq, Q, D]`` rotates at
    ``positions[b, K-Q+s]``; ``k [B, Hk, K, D]`` at ``positions[b, s]`` except
    Beacon keys - prefix rows ``sink <= s < K - len(roles)`` (history
    Beacons) and rows whose role is 1 or 2 - which keep their values.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    positions = np.asarray(positions, np.int64)
    roles = np.asarray(roles, np.int64)
    K, Q = k.shape[2], q.shape[2]
    prefix = K - len(roles)
    qo = rope_bf16(q, cos, sin, positions[:, None, K - Q:])
    ko = rope_bf16(k, cos, sin, positions[:, None, :])
    s = np.arange(K)
    role = np.zeros(K, np.int64)
    role[prefix:] = roles
    beacon = ((s < prefix) & (s >= sink)) | (role == 1) | (role == 2)
    ko[:, :, beacon] = k[:, :, beacon]
    return qo, ko


def flush_chunk(beacon_pages, raw_pages, beacon_table, raw_table, layout, block_size, key, value, key_latent,
                value_latent, raw_indices, lat_start, raw_start, raw_first, write_sink):
    """The page writes of one processed chunk for one sequence.

    Restates ``flush_memory`` (slimkv/vllm_plugin/paged_model.py:55-83) for
    the rows a chunk adds: Beacon latents at logical rows ``lat_start + j``
    (``BeaconPages.append``), raw K/V rows ``i >= raw_first`` at absolute raw
    positions ``raw_start + i`` (``RawPages.write``, pages
    ``[blocks, block_size, 2, Hkv, D]`` flattened to ``[blocks, block_size,
    2, Hkv*D]``) and, when ``write_sink``, the raw token at position 0 into
    the sink of the root Beacon page (``BeaconPages.write_sink``).
    ``key/value [n, kvd]`` are the chunk rows, ``key_latent/value_latent
    [n_beacon, R]``.
    """
    if len(key_latent):
        beacon_pages_append(beacon_pages, beacon_table, lat_start, key_latent, value_latent, layout)
    kvd = key.shape[-1]
    for i, row in enumerate(raw_indices):
        pos = raw_start + i
        if write_sink and pos == 0:
            root = beacon_table[0]
            beacon_pages[root, :kvd] = key[row]
            beacon_pages[root, kvd:2 * kvd] = value[row]
        if i < raw_first:
            continue
        blk = raw_table[pos // block_size]
        raw_pages[blk, pos % block_size, 0] = key[row]
        raw_pages[blk, pos % block_size, 1] = value[row]
