"""CPU restatement of one batched SlimKV decode layer (test infrastructure).

Used only as the timed CPU baseline by ``bench.py`` (``cpu_baseline`` and the
``--impl reference`` arm).  It follows the reference's eager fp32 decode
(slimkv/llama3/fa2_decode.py:77-166 with latent_decode.py:16-41 as the
attention) plus the Llama decoder layer around it (RMSNorm, the q/k/v and
Beacon projections, o_proj, SiLU-gated MLP), vectorised with numpy so that
the host's BLAS threads do the work.  Weights and caches are synthetic.
"""
import math
import os
import time

import numpy as np


def _rms(x, eps=1e-5):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)


def _rope(x, cos, sin, pos):
    """fp32 rotary of x [..., D] at positions pos (broadcast to x[..., 0])."""
    half = x.shape[-1] // 2
    c, s = cos[pos], sin[pos]
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * c + rot * s


def _softmax_attend(q, k, v, scale):
    """q [M, R], k [N, R], v [N, Rv] -> (out [M, Rv], lse [M])."""
    s = (q @ k.T) * scale
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    tot = p.sum(-1, keepdims=True)
    return (p @ v) / tot, (m + np.log(tot))[:, 0]


class CpuDecodeLayer:
    """One decoder layer's weights and caches for ``batch`` sequences."""

    def __init__(self, batch, history, tails, hidden=4096, heads=32, kv_heads=8, head_dim=128, rank=320,
                 intermediate=14336, sink=4, ratio=4, seed=0, std=0.02):
        rng = np.random.default_rng(seed)
        f32 = np.float32
        self.dims = (hidden, heads, kv_heads, head_dim, rank, intermediate)
        self.sink, self.ratio = sink, ratio
        w = lambda *s: rng.standard_normal(s, dtype=f32) * f32(std)
        qd, kvd = heads * head_dim, kv_heads * head_dim
        self.w_raw, self.w_beacon, self.w_o = w(qd + 2 * kvd, hidden), w(qd + 2 * rank, hidden), w(hidden, qd)
        self.uk = w(kvd, rank).reshape(kv_heads, head_dim, rank)
        self.uv = w(kvd, rank).reshape(kv_heads, head_dim, rank)
        self.w_gate_up, self.w_down = w(2 * intermediate, hidden), w(hidden, intermediate)
        self.history, self.tails = np.asarray(history), np.asarray(tails)
        nlat = self.history + self.tails // ratio + 1
        nraw = sink + self.tails + 1
        self.lat_k = [rng.standard_normal((n, rank), dtype=f32) * f32(1.3) for n in nlat]
        self.lat_v = [rng.standard_normal((n, rank), dtype=f32) * f32(1.3) for n in nlat]
        self.raw_k = [rng.standard_normal((n, kv_heads, head_dim), dtype=f32) * f32(1.3) for n in nraw]
        self.raw_v = [rng.standard_normal((n, kv_heads, head_dim), dtype=f32) * f32(1.3) for n in nraw]
        pos_max = int((sink + self.history + self.tails + self.tails // ratio).max()) + 4
        inv = 1.0 / (500000.0 ** (np.arange(0, head_dim, 2, dtype=f32) / head_dim))
        emb = np.concatenate([np.outer(np.arange(pos_max, dtype=f32), inv)] * 2, axis=-1)
        self.cos, self.sin = np.cos(emb).astype(f32), np.sin(emb).astype(f32)

    def forward(self, x):
        """x [B, 2, hidden] fp32 (raw row, Beacon row) -> updated x."""
        hidden, heads, kv_heads, d, rank, inter = self.dims
        B = x.shape[0]
        qd, kvd, group = heads * d, kv_heads * d, heads // kv_heads
        scale = 1.0 / math.sqrt(d)
        h = _rms(x)
        z_raw = h[:, 0] @ self.w_raw.T
        z_bcn = h[:, 1] @ self.w_beacon.T
        attn = np.zeros((B, 2, qd), np.float32)
        for b in range(B):
            t = int(self.tails[b])
            ins = (t + 1) % self.ratio == 0
            L = 1 + int(ins)
            pos = self.sink + int(self.history[b]) + t + t // self.ratio
            q = z_raw[b, :qd][None] if not ins else np.stack([z_raw[b, :qd], z_bcn[b, :qd]])
            q = _rope(q.reshape(L, heads, d), self.cos, self.sin, (pos + np.arange(L))[:, None])
            k_new = _rope(z_raw[b, qd:qd + kvd].reshape(kv_heads, d), self.cos, self.sin, pos)
            rk = np.concatenate([self.raw_k[b][:-1], k_new[None]])
            rv = np.concatenate([self.raw_v[b][:-1], z_raw[b, qd + kvd:].reshape(1, kv_heads, d)])
            n_lat = len(self.lat_k[b]) - (0 if ins else 1)
            lk, lv = self.lat_k[b][:n_lat], self.lat_v[b][:n_lat]
            for g in range(kv_heads):
                qg = q[:, g * group:(g + 1) * group].reshape(L * group, d)
                ro, rl = _softmax_attend(qg, rk[:, g], rv[:, g], scale)
                ql = qg @ self.uk[g]                                        # q-absorb
                lo, ll = _softmax_attend(ql, lk, lv, scale)
                if ins:                                                     # raw query excludes the Beacon
                    lo0, ll0 = _softmax_attend(ql[:group], lk[:-1], lv[:-1], scale)
                    lo[:group], ll[:group] = lo0, ll0
                up = lo @ self.uv[g].T
                tot = np.logaddexp(rl, ll)
                out = np.exp(rl - tot)[:, None] * ro + np.exp(ll - tot)[:, None] * up
                attn[b, :L, g * group * d:(g + 1) * group * d] = out.reshape(L, group * d)
        x = x + attn @ self.w_o.T
        h2 = _rms(x)
        gu = h2 @ self.w_gate_up.T
        a = gu[..., :inter] / (1 + np.exp(-gu[..., :inter])) * gu[..., inter:]
        return x + a @ self.w_down.T


def time_decode_step(batch=16, layers=32, history=8192, seed=1234, repeats=2, vocab=128256, hidden=4096):
    """Seconds of one full decode step, from a timed single-layer sample.

    One decoder layer is timed ``repeats`` times for the whole batch and
    scaled by ``layers``; the vocabulary projection of the batch is timed once
    on a slice and scaled to the full vocabulary.  Returns ``(seconds,
    threads, sample description)``.
    """
    rng = np.random.default_rng(seed)
    tails = rng.integers(0, 1024, size=batch)
    layer = CpuDecodeLayer(batch, np.full(batch, history), tails, hidden=hidden)
    x = rng.standard_normal((batch, 2, hidden), dtype=np.float32)
    layer.forward(x)
    t0 = time.perf_counter()
    for _ in range(repeats):
        layer.forward(x)
    per_layer = (time.perf_counter() - t0) / repeats
    head = rng.standard_normal((vocab // 8, hidden), dtype=np.float32) * np.float32(0.02)
    t0 = time.perf_counter()
    _ = _rms(x[:, 0]) @ head.T
    lm = (time.perf_counter() - t0) * 8
    threads = len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else os.cpu_count()
    sample = (f'1 of {layers} decoder layers x {repeats} repeats for batch {batch} at {history} latents + '
              f'raw tail U{{0..1023}} (scaled x{layers}), vocab projection on 1/8 of the rows (scaled x8)')
    return per_layer * layers + lm, threads, sample
