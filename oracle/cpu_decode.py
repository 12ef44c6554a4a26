"""CPU restatement of one batched SlimKV decode layer (test infrastructure).

The timed CPU fallback of ``bench.py`` when the reference package is not
installed beside the repository, and a checker pinned to the reference's
``decode`` goldens (``tests/test_cpu_decode_port.py``).  It follows the
reference's eager fp32 decode (slimkv/llama3/fa2_decode.py:77-166 with
latent_decode.py:16-41 as the attention): projections of the raw row and of
an inserted Beacon row, RoPE of the query rows and of the sink + open-window
raw keys at their absolute positions (recomputed every step, as the
reference does), raw and latent attention merged by LSE, the K/V
up-projection biases, ``o_proj``; and the Llama decoder layer around it
(RMSNorm, SiLU-gated MLP) for whole-step timing.  numpy float32; the host's
BLAS threads do the matrix work.
"""
import math
import os
import time

import numpy as np

from .rope import rope_tables

# Llama-3.1-8B rotary setup (config.json of the checkpoint): theta 500000 with
# Llama-3 frequency scaling.
LLAMA3_THETA = 500000.0
LLAMA3_SCALING = dict(factor=8.0, original_max_position_embeddings=8192, low_freq_factor=1.0, high_freq_factor=4.0)


def _rms(x, eps=1e-5):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)


def _rope(x, cos, sin, pos):
    """fp32 rotary of x [..., D] at positions pos (broadcast to x[..., 0]);
    rotate_half convention (slimkv/modeling_utils.py rotate_half)."""
    half = x.shape[-1] // 2
    c, s = cos[pos], sin[pos]
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * c + rot * s


def _softmax_attend(q, k, v, scale):
    """q [M, R], k [N, R], v [N, Rv] -> (out [M, Rv], lse [M]); N may be 0."""
    if k.shape[0] == 0:
        return np.zeros((q.shape[0], v.shape[1]), np.float32), np.full(q.shape[0], -np.inf, np.float32)
    s = (q @ k.T) * np.float32(scale)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    tot = p.sum(-1, keepdims=True)
    return (p @ v) / tot, (m + np.log(tot))[:, 0]


class CpuDecodeLayer:
    """One decoder layer's weights and the caches of ``len(seqs)`` sequences.

    ``weights`` uses the names of ``tests/golden/cases.config1_layer``:
    ``q_proj``, ``k_proj``, ``v_proj``, ``o_proj``, ``beacon_q_proj``,
    ``k_down``, ``v_down``, ``k_up`` [Hkv*D, R], ``v_up`` (nn.Linear
    ``[out, in]`` layout) and optional ``q_bias``, ``k_bias``, ``v_bias``,
    ``o_bias``, ``beacon_q_bias``, ``k_up_bias``, ``v_up_bias``; ``gate_up``
    [2I, hidden] and ``down`` for the MLP of ``forward``.

    Each sequence is a dict: ``sink_k`` / ``sink_v`` [S, Hkv, D] and
    ``raw_k`` / ``raw_v`` [T, Hkv, D] pre-RoPE, ``raw_pos`` [T] (absolute
    positions of the open window's raw tokens: window index + sink + history
    latents), ``lat_k`` / ``lat_v`` [n, R] (history + open-window Beacons) and
    ``position`` (this step's raw token).
    """

    def __init__(self, weights, seqs, heads, kv_heads, head_dim, cos, sin):
        self.w = {k: np.ascontiguousarray(v, np.float32) for k, v in weights.items()}
        self.seqs = seqs
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.cos, self.sin = cos, sin
        d = head_dim
        self.uk = self.w['k_up'].reshape(kv_heads, d, -1)           # [g] : [D, R]
        self.uv = self.w['v_up'].reshape(kv_heads, d, -1)

    def _lin(self, x, name, bias=None):
        y = x @ self.w[name].T
        if bias in self.w:
            y = y + self.w[bias]
        return y

    def attend(self, h, lengths):
        """Attention output after ``o_proj`` for the attention input rows ``h``
        [B, 2, hidden] (row 1 = the Beacon row where ``lengths[b] == 2``).

        Returns ``(out [B, 2, hidden], new_lat_k [B, R], new_lat_v [B, R])``
        (rows past ``lengths[b]`` and the latents of sequences without a
        Beacon are zero)."""
        heads, kv_heads, d = self.heads, self.kv_heads, self.head_dim
        B = h.shape[0]
        qd, kvd, group = heads * d, kv_heads * d, heads // kv_heads
        scale = 1.0 / math.sqrt(d)
        raw_rows = h[:, 0]
        q_raw = self._lin(raw_rows, 'q_proj', 'q_bias')
        k_new = self._lin(raw_rows, 'k_proj', 'k_bias').reshape(B, kv_heads, d)
        v_new = self._lin(raw_rows, 'v_proj', 'v_bias').reshape(B, kv_heads, d)
        ins = np.asarray(lengths) == 2
        q_bcn = np.zeros_like(q_raw)
        lk_new = np.zeros((B, self.uk.shape[2]), np.float32)
        lv_new = np.zeros((B, self.uv.shape[2]), np.float32)
        if ins.any():
            hb = h[ins, 1]
            q_bcn[ins] = self._lin(hb, 'beacon_q_proj', 'beacon_q_bias')
            lk_new[ins] = self._lin(hb, 'k_down')
            lv_new[ins] = self._lin(hb, 'v_down')
        attn = np.zeros((B, 2, qd), np.float32)
        kb = self.w.get('k_up_bias')
        vb = self.w.get('v_up_bias')
        for b, sq in enumerate(self.seqs):
            L = 2 if ins[b] else 1
            pos = int(sq['position'])
            q = q_raw[b][None] if L == 1 else np.stack([q_raw[b], q_bcn[b]])
            q = _rope(q.reshape(L, heads, d), self.cos, self.sin, (pos + np.arange(L))[:, None])
            kpos = np.concatenate([np.arange(len(sq['sink_k'])), sq['raw_pos'], [pos]]).astype(np.int64)
            rk = _rope(np.concatenate([sq['sink_k'], sq['raw_k'], k_new[b][None]]), self.cos, self.sin,
                       kpos[:, None])
            rv = np.concatenate([sq['sink_v'], sq['raw_v'], v_new[b][None]])
            lk, lv = sq['lat_k'], sq['lat_v']
            if L == 2:
                lk = np.concatenate([lk, lk_new[b][None]])
                lv = np.concatenate([lv, lv_new[b][None]])
            for g in range(kv_heads):
                qg = q[:, g * group:(g + 1) * group].reshape(L * group, d)
                ro, rl = _softmax_attend(qg, rk[:, g], rv[:, g], scale)
                ql = qg @ self.uk[g]                                        # query absorbed into latent space
                lo, ll = _softmax_attend(ql, lk, lv, scale)
                if L == 2:                                                  # the raw query excludes the new Beacon
                    lo0, ll0 = _softmax_attend(ql[:group], lk[:-1], lv[:-1], scale)
                    lo[:group], ll[:group] = lo0, ll0
                if kb is not None:
                    ll = ll + (qg @ kb[g * d:(g + 1) * d]) * np.float32(scale)
                up = lo @ self.uv[g].T
                if vb is not None:
                    up = up + vb[g * d:(g + 1) * d]
                tot = np.logaddexp(rl, ll)
                out = np.exp(rl - tot)[:, None] * ro + np.exp(ll - tot)[:, None] * up
                attn[b, :L, g * group * d:(g + 1) * group * d] = out.reshape(L, group * d)
        out = self._lin(attn, 'o_proj', 'o_bias')
        for b in range(B):
            if not ins[b]:
                out[b, 1] = 0
        return out, lk_new, lv_new

    def forward(self, x, lengths):
        """Decoder layer: x [B, 2, hidden] fp32 residual stream -> updated x."""
        a, _, _ = self.attend(_rms(x), lengths)
        x = x + a
        gu = _rms(x) @ self.w['gate_up'].T
        inter = gu.shape[-1] // 2
        act = gu[..., :inter] / (1 + np.exp(-gu[..., :inter])) * gu[..., inter:]
        return x + act @ self.w['down'].T

    @classmethod
    def synthetic(cls, history, tails, hidden=4096, heads=32, kv_heads=8, head_dim=128, rank=320,
                  intermediate=14336, sink=4, ratio=4, seed=0, std=0.02):
        """Random N(0, std) weights and N(0, 1.3^2) caches for sequences at
        ``history`` latents and open-window raw tails ``tails`` (each decoding
        raw token ``tails[b]``; a Beacon is inserted when ``(t + 1) % ratio
        == 0``).  Returns ``(layer, lengths)``."""
        rng = np.random.default_rng(seed)
        f32 = np.float32
        w = lambda *s: rng.standard_normal(s, dtype=f32) * f32(std)
        qd, kvd = heads * head_dim, kv_heads * head_dim
        weights = dict(q_proj=w(qd, hidden), k_proj=w(kvd, hidden), v_proj=w(kvd, hidden), o_proj=w(hidden, qd),
                       beacon_q_proj=w(qd, hidden), k_down=w(rank, hidden), v_down=w(rank, hidden),
                       k_up=w(kvd, rank), v_up=w(kvd, rank), gate_up=w(2 * intermediate, hidden),
                       down=w(hidden, intermediate))
        seqs, lengths = [], []
        r = lambda *s: rng.standard_normal(s, dtype=f32) * f32(1.3)
        for n_hist, t in zip(np.broadcast_to(history, np.shape(tails)), tails):
            t, n_hist = int(t), int(n_hist)
            idx = np.arange(t) + np.arange(t) // ratio
            nl = n_hist + t // ratio
            seqs.append(dict(sink_k=r(sink, kv_heads, head_dim), sink_v=r(sink, kv_heads, head_dim),
                             raw_k=r(t, kv_heads, head_dim), raw_v=r(t, kv_heads, head_dim),
                             raw_pos=idx + sink + n_hist, lat_k=r(nl, rank), lat_v=r(nl, rank),
                             position=sink + n_hist + t + t // ratio))
            lengths.append(2 if (t + 1) % ratio == 0 else 1)
        pos_max = max(s['position'] for s in seqs) + 2
        cos, sin = rope_tables(head_dim, LLAMA3_THETA, pos_max, LLAMA3_SCALING)
        return cls(weights, seqs, heads, kv_heads, head_dim, cos, sin), np.array(lengths)


def time_decode_step(batch=16, layers=32, history=8192, seed=1234, repeats=2, vocab=128256, hidden=4096):
    """Seconds of one full decode step, from a timed single-layer sample.

    One decoder layer is timed ``repeats`` times for the whole batch and
    scaled by ``layers``; the vocabulary projection of the batch is timed once
    on a slice and scaled to the full vocabulary.  Returns ``(seconds,
    threads, sample description)``.
    """
    rng = np.random.default_rng(seed)
    tails = rng.integers(0, 1024, size=batch)
    layer, lengths = CpuDecodeLayer.synthetic(history, tails, hidden=hidden)
    x = rng.standard_normal((batch, 2, hidden), dtype=np.float32)
    layer.forward(x, lengths)
    t0 = time.perf_counter()
    for _ in range(repeats):
        layer.forward(x, lengths)
    per_layer = (time.perf_counter() - t0) / repeats
    head = rng.standard_normal((vocab // 8, hidden), dtype=np.float32) * np.float32(0.02)
    t0 = time.perf_counter()
    _ = _rms(x[:, 0]) @ head.T
    lm = (time.perf_counter() - t0) * 8
    threads = len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else os.cpu_count()
    sample = (f'numpy restatement: 1 of {layers} decoder layers x {repeats} repeats for batch {batch} at {history} '
              f'latents + raw tail U{{0..1023}} (scaled x{layers}), vocab projection on 1/8 of the rows (scaled x8)')
    return per_layer * layers + lm, threads, sample
