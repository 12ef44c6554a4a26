"""Parity of one decode layer at the BASELINE configurations' shapes.

The smaller parity cases (``test_gpu_decode.py``) exercise every branch of
the kernels; these run the launches the bench times, with the work plans
those shapes produce, against the oracle (float64 restatement of the
reference's eager latent path, pinned to the reference's goldens):

* config 2 — Llama-3.1-8B r4 / t4: 16 sequences at 32768 tokens (8192
  history latents plus the open window's), raw tails U{0..1023}, mixed
  insertion rows, dense native cache, the default persistent plan over every
  SM (segments split over many CTAs, CTAs spanning segments);
* config 3 — r8 / t8 (ranks 160), 256 sequences with contexts in [2048,
  131072] in shuffled Beacon pages: the full launch runs, and 24 sequences
  spread over the length range are checked against the oracle;
* config 5 — Qwen2.5-14B geometry (40 / 8 heads, q/k/v-style biases on the
  up-projections, r2 ranks 512) at 32768 latents, the split-KV route.

fp32 output mode, so the bar is the norm-wise 2e-3 of BASELINE.json (plus the
reference GPU validation's element-wise tolerance); cache writes bit-exact.
"""
import numpy as np
import pytest
import torch

from cases import decode_case
from test_gpu_decode import check, oracle_rows, run_fused, tables
from gpu_util import assert_attention_close, to_bf16

pytestmark = pytest.mark.gpu


def test_config2_shape_full_plan():
    c = decode_case(2002, batch=16, length=2, history=8192, tail=1023, ragged=False)
    rng = np.random.default_rng(7)
    # Every sequence at its own raw tail (the bench draws U{0..1023}).
    tails = rng.integers(0, 1024, size=16)
    query_len = np.array([2 if (t + 1) % 4 == 0 else 1 for t in tails])
    query_len[:4] = 2                                  # at least a few insertion rows
    c['n_raw'] = 4 + tails + 1
    c['n_lat'] = 8192 + tails // 4 + (query_len - 1)
    win = tails // 4
    for b in range(16):
        t = int(tails[b])
        current = 4 + 8192 + t + int(win[b])
        c['qpos'][b] = current + np.arange(2)
        idx = np.arange(t) + np.arange(t) // 4
        c['kpos'][b, :c['n_raw'][b]] = np.concatenate([np.arange(4), idx + 4 + 8192, [current]])
    err = check(c, query_len, run_fused(c, query_len, fp32=True))
    assert err <= 2e-3


def test_config5_shape_qwen_rank512():
    c = decode_case(2005, batch=2, length=2, history=32768, tail=700, heads=40, kv_heads=8, rk=512, rv=512, bias=True)
    query_len = np.array([2, 1])
    check(c, query_len, run_fused(c, query_len, fp32=True, positions=65536), positions=65536)


def test_config3_shape_paged_r8_large_batch():
    """256 requests, ranks 160, t8 Beacons, contexts across [2048, 131072] in
    Beacon pages (96 slots per page): one launch, 24 rows checked."""
    from slimkv_b200 import kernels, pages as P, _lib
    rng = np.random.default_rng(2003)
    B, H, Hkv, D, R, ratio = 256, 32, 8, 128, 160, 8
    ctx = rng.integers(2048, 131073, size=B)
    tails = ctx % 1024
    hist = ctx // 1024 * (1024 // ratio)
    query_len = np.where((tails + 1) % ratio == 0, 2, 1)
    n_lat = hist + tails // ratio + (query_len - 1)
    n_raw = 4 + tails + 1
    cos, sin, cos_t, sin_t = tables(32768)
    dev = torch.device('cuda', 0)
    layout = P.BeaconPageLayout(768, ratio, R, R, Hkv * D)
    per_seq = (n_lat + layout.slots - 1) // layout.slots
    perm = rng.permutation(int(per_seq.sum()))
    table = np.zeros((B, per_seq.max()), np.int32)
    at = 0
    for b in range(B):
        table[b, :per_seq[b]] = perm[at:at + per_seq[b]]
        at += per_seq[b]
    table_t = torch.from_numpy(table).to(dev)
    pages = torch.zeros(len(perm), layout.page_elements, dtype=torch.bfloat16, device=dev)
    # Latents: one random block per sequence length, written through the
    # page drop-in (bit-exact with the reference's BeaconPages.append).
    lat = []
    for b in range(B):
        k = to_bf16(rng.standard_normal((int(n_lat[b]), R), dtype=np.float32) * 1.3)
        v = to_bf16(rng.standard_normal((int(n_lat[b]), R), dtype=np.float32) * 1.3)
        P.beacon_append(pages, layout, table_t[b:b + 1], [0], k[None], v[None])
        lat.append((k, v))
    raw_cap = 1088
    raw_k = to_bf16(rng.standard_normal((B, raw_cap, Hkv, D), dtype=np.float32) * 1.3)
    raw_v = to_bf16(rng.standard_normal((B, raw_cap, Hkv, D), dtype=np.float32) * 1.3)
    q = to_bf16(rng.standard_normal((B, 2, H, D), dtype=np.float32) * 1.3)
    uk = to_bf16(rng.standard_normal((Hkv * D, R), dtype=np.float32) * 0.05)
    uv = to_bf16(rng.standard_normal((Hkv * D, R), dtype=np.float32) * 0.05)
    qpos = np.stack([4 + hist + tails + tails // ratio + l for l in range(2)], 1).astype(np.int32)
    i32 = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.int32)).to(dev)
    out = torch.zeros(B, 2, H * D, dtype=torch.float32, device=dev)
    _lib.device_status(clear=True)
    # The cache already holds this step's rows (no appends): keys are taken as
    # rotated as stored, which the oracle reproduces with identity positions.
    kernels.latent_decode(q=q, raw_k_rot=raw_k, raw_v=raw_v, lat_pages=(pages, layout, table_t), raw_len=i32(n_raw),
                          latent_len=i32(n_lat), query_len=i32(query_len), qpos=i32(qpos), uk=uk, uv=uv, cos=cos_t,
                          sin=sin_t, out=out, latent_len_max=int(n_lat.max()), raw_len_max=raw_cap)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    assert torch.isfinite(out).all()
    order = np.argsort(ctx)
    rows = order[np.linspace(0, B - 1, 24).astype(int)]
    f = lambda t: t.float().cpu().numpy()
    qn, rkn, rvn, ukn, uvn = f(q), f(raw_k), f(raw_v), f(uk), f(uv)
    for b in rows:
        L, nr = int(query_len[b]), int(n_raw[b])
        # Raw keys are stored rotated: rotating the oracle's copy by position
        # 0 (cos 1, sin 0) leaves them unchanged.
        kpos = np.zeros((1, nr), np.int64)
        ref = oracle.latent_decode_attention(qn[b:b + 1, :L], rkn[b:b + 1, :nr], rvn[b:b + 1, :nr],
                                             f(lat[b][0])[None], f(lat[b][1])[None], ukn, uvn, cos, sin,
                                             qpos[b:b + 1, :L], kpos, L - 1)['out']
        assert_attention_close(out[b:b + 1, :L], ref)


import oracle  # noqa: E402  (test infrastructure: the checker)
