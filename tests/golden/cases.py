"""Seeded synthetic inputs shared by the golden generator and the tests.

Everything is built with numpy's ``default_rng`` so that the fixture script,
the CPU oracle tests and the GPU parity tests see bit-identical inputs.
No benchmark dataset is involved: the reference's LongBench runs are stood in
for by random tensors with the BASELINE geometries.
"""
import numpy as np

LLAMA8B = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, theta=500000.0,
               scaling=dict(factor=8.0, original_max_position_embeddings=8192,
                            low_freq_factor=1.0, high_freq_factor=4.0),
               max_positions=131072)


def _bf16(x):
    from oracle.bf16 import round_bf16
    return round_bf16(np.asarray(x, np.float32))


def attention_case(seed, batch, queries, heads, kv_heads, keys, dk, dv, causal,
                   bf16=True, scale=None, lengths=None):
    """q/k/v for one grouped decode attention call (BSHD, values as fp32)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((batch, queries, heads, dk), dtype=np.float32) * 0.3
    k = rng.standard_normal((batch, keys, kv_heads, dk), dtype=np.float32) * 0.3
    v = rng.standard_normal((batch, keys, kv_heads, dv), dtype=np.float32)
    if bf16:
        q, k, v = _bf16(q), _bf16(k), _bf16(v)
    return dict(q=q, k=k, v=v, scale=scale if scale is not None else 1.0 / np.sqrt(128.0),
                causal=causal, lengths=lengths)


def decode_case(seed, batch, length, history, tail, sink=4, heads=32, kv_heads=8,
                head_dim=128, rk=320, rv=320, bias=False, ratio=4, window_latents=None,
                ragged=False):
    """Attention-level inputs of one decode step over the compressed cache.

    ``history`` completed-window latents, ``tail`` raw tokens of the open
    window (Beacons interleaved every ``ratio`` raw tokens), ``sink`` sinks,
    ``length`` = 1 + inserted Beacon.  With ``ragged`` each batch row draws its
    own history and tail below the given maxima.  Values are bf16-rounded.
    Magnitudes follow projections of unit-variance hidden states through
    N(0, 0.02) weights (``|x| ~ 0.02 * sqrt(4096) = 1.3``).
    """
    rng = np.random.default_rng(seed)
    if ragged:
        hist = rng.integers(max(history // 2, 0), history + 1, size=batch)
        tails = rng.integers(0, tail + 1, size=batch)
    else:
        hist = np.full(batch, history)
        tails = np.full(batch, tail)
    win = tails // ratio if window_latents is None else np.full(batch, window_latents)
    size = length - 1
    n_lat = hist + win + size                      # latent rows incl. new Beacon
    n_raw = sink + tails + 1                       # sink + tail + current raw token
    mag = 1.3
    q = _bf16(rng.standard_normal((batch, length, heads, head_dim), dtype=np.float32) * mag)
    raw_k = _bf16(rng.standard_normal((batch, n_raw.max(), kv_heads, head_dim), dtype=np.float32) * mag)
    raw_v = _bf16(rng.standard_normal((batch, n_raw.max(), kv_heads, head_dim), dtype=np.float32) * mag)
    lat_k = _bf16(rng.standard_normal((batch, max(n_lat.max(), 1), rk), dtype=np.float32) * mag)
    lat_v = _bf16(rng.standard_normal((batch, max(n_lat.max(), 1), rv), dtype=np.float32) * mag)
    uk = _bf16(rng.standard_normal((kv_heads * head_dim, rk), dtype=np.float32) * 0.05)
    uv = _bf16(rng.standard_normal((kv_heads * head_dim, rv), dtype=np.float32) * 0.05)
    bk = _bf16(rng.standard_normal(kv_heads * head_dim, dtype=np.float32) * 0.02) if bias else None
    bv = _bf16(rng.standard_normal(kv_heads * head_dim, dtype=np.float32) * 0.02) if bias else None
    # Compressed positions (slimkv/llama3/fa2_decode.py:127-131): the current
    # raw token sits after sinks, history and the interleaved open window.
    qpos = np.zeros((batch, length), np.int64)
    kpos = np.zeros((batch, n_raw.max()), np.int64)
    for b in range(batch):
        t = int(tails[b])
        current = sink + hist[b] + t + int(win[b])
        qpos[b] = current + np.arange(length)
        idx = np.arange(t) + np.arange(t) // ratio
        kpos[b, :n_raw[b]] = np.concatenate([np.arange(sink), idx + sink + hist[b], [current]])
    return dict(q=q, raw_k=raw_k, raw_v=raw_v, lat_k=lat_k, lat_v=lat_v, uk=uk, uv=uv,
                bk=bk, bv=bv, qpos=qpos, kpos=kpos, n_lat=n_lat.astype(np.int64),
                n_raw=n_raw.astype(np.int64), size=size, sink=sink, hist=hist, tails=tails,
                win=win, heads=heads, kv_heads=kv_heads, head_dim=head_dim, rk=rk, rv=rv)


def config1_layer(batch=1, length=1, history=2048, sink=4, tail=0, rank=320, seed_w=0,
                  seed_h=1, hidden=4096, heads=32, kv_heads=8, head_dim=128, bias=False):
    """one Llama-3.1-8B-geometry layer, fp32, on the CPU.

    Weights ~ N(0, 0.02) from ``default_rng(seed_w)``; hidden states ~ N(0, 1)
    from ``default_rng(seed_h)``.  The cache is produced by the layer's own
    projections of hidden states: pre-RoPE sink/raw K and V through
    ``k_proj``/``v_proj`` and Beacon latents through the down projections.
    """
    rw = np.random.default_rng(seed_w)

    def w(out, inp):
        return rw.standard_normal((out, inp), dtype=np.float32) * np.float32(0.02)

    kvd = kv_heads * head_dim
    weights = dict(q_proj=w(heads * head_dim, hidden), k_proj=w(kvd, hidden),
                   v_proj=w(kvd, hidden), o_proj=w(hidden, heads * head_dim),
                   beacon_q_proj=w(heads * head_dim, hidden), k_down=w(rank, hidden),
                   k_up=w(kvd, rank), v_down=w(rank, hidden), v_up=w(kvd, rank))
    if bias:
        for name, n in [('q_bias', heads * head_dim), ('k_bias', kvd), ('v_bias', kvd),
                        ('o_bias', hidden), ('beacon_q_bias', heads * head_dim),
                        ('k_up_bias', kvd), ('v_up_bias', kvd)]:
            weights[name] = rw.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    rh = np.random.default_rng(seed_h)
    x = rh.standard_normal((batch, length, hidden), dtype=np.float32)
    hs = rh.standard_normal((batch, sink + tail, hidden), dtype=np.float32)
    hb = rh.standard_normal((batch, history + tail // 4, hidden), dtype=np.float32)

    def lin(h, name, bname=None):
        y = h @ weights[name].T
        if bias and bname:
            y = y + weights[bname]
        return y.astype(np.float32)

    raw_k = lin(hs, 'k_proj', 'k_bias').reshape(batch, sink + tail, kv_heads, head_dim)
    raw_v = lin(hs, 'v_proj', 'v_bias').reshape(batch, sink + tail, kv_heads, head_dim)
    lat_k = lin(hb, 'k_down')
    lat_v = lin(hb, 'v_down')
    return dict(weights=weights, hidden=x, sink_k=raw_k[:, :sink], sink_v=raw_v[:, :sink],
                tail_k=raw_k[:, sink:], tail_v=raw_v[:, sink:], hist_k=lat_k[:, :history],
                hist_v=lat_v[:, :history], win_k=lat_k[:, history:], win_v=lat_v[:, history:],
                batch=batch, length=length, history=history, sink=sink, tail=tail, rank=rank,
                hidden_size=hidden, heads=heads, kv_heads=kv_heads, head_dim=head_dim, bias=bias)


# A two-layer SlimKV Llama with the Llama-3.1-8B attention geometry (32 / 8
# heads, head_dim 128, r4 ranks 320 / 320) but a small vocabulary, a narrow
# MLP and a 64-token Beacon window, so that the reference model runs prefill
# plus decode across a window rollover on the CPU in seconds.
TINY_MODEL = dict(vocab=256, hidden=4096, intermediate=512, layers=2, heads=32, kv_heads=8, head_dim=128,
                  rank=320, window=64, ratio=4, sink=4, theta=500000.0, rms_eps=1e-5,
                  prefill=212, steps=60, seed=2024)


def tiny_model_weights(spec=TINY_MODEL):
    """bf16-representable weights (as fp32 arrays) of the tiny model, keyed by
    the reference's parameter names; linear weights ~ N(0, 0.02) (lm_head
    N(0, 0.008)), embeddings ~ N(0, 1), norm weights ~ 1 + N(0, 0.1)."""
    import torch                      # exact round-to-nearest-even, faster than numpy for 139M values
    rng = np.random.default_rng(spec['seed'])
    H, I, V, R = spec['hidden'], spec['intermediate'], spec['vocab'], spec['rank']
    qd, kvd = spec['heads'] * spec['head_dim'], spec['kv_heads'] * spec['head_dim']

    def _bf16(x):
        return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).float().numpy()

    def w(*shape, std=0.02):
        return _bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    out = {'model.embed_tokens.weight': w(V, H, std=1.0), 'model.beacon_embed_tokens.weight': w(1, H, std=1.0)}
    for i in range(spec['layers']):
        p = f'model.layers.{i}.'
        out.update({
            p + 'self_attn.q_proj.weight': w(qd, H), p + 'self_attn.k_proj.weight': w(kvd, H),
            p + 'self_attn.v_proj.weight': w(kvd, H), p + 'self_attn.o_proj.weight': w(H, qd),
            p + 'self_attn.beacon_q_proj.weight': w(qd, H),
            p + 'self_attn.beacon_k_down_proj.weight': w(R, H), p + 'self_attn.beacon_k_up_proj.weight': w(kvd, R),
            p + 'self_attn.beacon_v_down_proj.weight': w(R, H), p + 'self_attn.beacon_v_up_proj.weight': w(kvd, R),
            p + 'mlp.gate_proj.weight': w(I, H), p + 'mlp.up_proj.weight': w(I, H), p + 'mlp.down_proj.weight': w(H, I),
            p + 'input_layernorm.weight': _bf16(1 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.1)),
            p + 'post_attention_layernorm.weight': _bf16(1 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))})
    out['model.norm.weight'] = _bf16(1 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
    # Logits of std ~0.5, the scale of the reference test suite's tiny model
    # (hidden 32, weights N(0, 0.1)), so that a bf16 model's rounding noise
    # stays well inside the 2e-2 logits bar.
    out['lm_head.weight'] = w(V, H, std=0.008)
    return out


def tiny_model_tokens(spec=TINY_MODEL):
    """Prefill token ids and the tokens fed at each decode step."""
    rng = np.random.default_rng(spec['seed'] + 1)
    return (rng.integers(0, spec['vocab'], size=spec['prefill']),
            rng.integers(0, spec['vocab'], size=spec['steps']))
