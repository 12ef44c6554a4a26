"""The reconstruct decode backend: Beacon K/V rebuilt from latents, then
ordinary attention (reference ``reconstruction_attention``,
tools/benchmark/context_decode_runtime.py:298-344, on
``ReconstructionCache.materialize``, slimkv/llama3/memory.py:26-48).

CPU: the oracle's ``materialize`` against the reference's own bf16
``nn.Linear`` outputs (``tests/golden/reconstruct_golden.npz``, made by
``make_golden.py --only reconstruct``), and the reconstruct oracle against
the latent-path oracle (the same attention up to the bf16 rounding of the
rebuilt keys and values).  GPU: ``slimkv_reconstruct_kv`` against both, and
the backend's attention output against the reconstruct oracle.
"""
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle.bf16 import bf16_bits, from_bf16_bits
from oracle.decode import latent_decode_attention
from oracle.reconstruct import materialize, reconstruct_decode_attention
from cases import decode_case, LLAMA8B

GOLDEN = Path(__file__).parent / 'golden' / 'reconstruct_golden.npz'


def _f(x):
    return from_bf16_bits(np.asarray(x).view(np.uint16))


def _ulps(a_bits, b_bits):
    def ordered(x):
        x = np.asarray(x, np.uint16).astype(np.int32)
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), x + 0x8000)
    return np.abs(ordered(a_bits) - ordered(b_bits))


def _golden_cases():
    d = np.load(GOLDEN)
    for name in ('qwen_r2', 'llama_r4'):
        for kind in 'kv':
            b = d.get(f'{name}_b_{kind}')
            yield (name, kind, _f(d[f'{name}_lat_{kind}']), _f(d[f'{name}_w_{kind}']),
                   None if b is None else _f(b), d[f'{name}_full_{kind}'].view(np.uint16))


def assert_near_bits(got, want, max_frac):
    """Within one bf16 ulp, or - where the dot product cancels to a value far
    below its terms, so that fp32 accumulation order decides more bits -
    within 1e-5 x max|want|; at most ``max_frac`` of the elements differ."""
    d = _ulps(got, want)
    g, w = from_bf16_bits(got), from_bf16_bits(want)
    far = (d > 1) & (np.abs(g - w) > 1e-5 * np.abs(w).max())
    assert not far.any(), f'{far.sum()} elements beyond one ulp, first at {np.argwhere(far)[:3].tolist()}'
    assert (d > 0).mean() <= max_frac, f'{(d > 0).mean():.3%} of elements differ'


def test_materialize_matches_reference_linear():
    """bf16(latent . W^T + b) with one rounding: the reference's bf16 Linear
    on CPU gives the same bits except where its fp32 accumulation order
    tips a rounding (under 0.1% of the elements)."""
    for name, kind, lat, w, b, want in _golden_cases():
        assert_near_bits(bf16_bits(materialize(lat, w, b)).reshape(want.shape), want, 1e-3)


def test_reconstruct_oracle_agrees_with_latent_oracle():
    """Both backends attend over the same keys; they differ only by the bf16
    rounding of the rebuilt keys and values."""
    cos, sin = oracle.rope_tables(128, LLAMA8B['theta'], 16384, LLAMA8B['scaling'])
    for length in (1, 2):
        c = decode_case(91 + length, batch=1, length=length, history=200, tail=30, bias=True)
        nr, nl = int(c['n_raw'][0]), int(c['n_lat'][0])
        args = (c['q'], c['raw_k'][:, :nr], c['raw_v'][:, :nr], c['lat_k'][:, :nl], c['lat_v'][:, :nl], c['uk'],
                c['uv'], cos, sin, c['qpos'], c['kpos'][:, :nr], length - 1)
        rec = reconstruct_decode_attention(*args, uk_bias=c['bk'], uv_bias=c['bv'])
        lat = latent_decode_attention(*args, uk_bias=c['bk'], uv_bias=c['bv'])
        err = np.linalg.norm(rec['out'] - lat['out']) / np.linalg.norm(lat['out'])
        assert err < 1e-2, err


# ---- GPU ----------------------------------------------------------------------

def _cuda():
    import torch
    return torch


@pytest.mark.gpu
def test_reconstruct_kv_matches_reference_golden():
    torch = _cuda()
    from gpu_util import to_bf16
    from slimkv_b200.reconstruct import reconstruct_kv
    d = {}
    for name, kind, lat, w, b, want in _golden_cases():
        d.setdefault(name, {})[kind] = (lat, w, b, want)
    for name, kv in d.items():
        (lk, wk, bk, want_k), (lv, wv, bv, want_v) = kv['k'], kv['v']
        B, n, R = lk.shape
        lat = to_bf16(np.concatenate([lk, lv], axis=-1))
        key = torch.zeros(B, n, want_k.shape[2], want_k.shape[3], dtype=torch.bfloat16, device='cuda')
        value = torch.zeros_like(key)
        reconstruct_kv(lat[..., :R], lat[..., R:], to_bf16(wk), to_bf16(wv), key, value, n,
                       None if bk is None else to_bf16(bk), None if bv is None else to_bf16(bv))
        torch.cuda.synchronize()
        for got, want in ((key, want_k), (value, want_v)):
            assert_near_bits(got.view(torch.int16).cpu().numpy().view(np.uint16), want, 5e-3)


@pytest.mark.gpu
@pytest.mark.parametrize('rank,kv_heads,batch,counted', [(512, 8, 3, False), (320, 8, 2, False), (160, 8, 1, False),
                                                         (64, 2, 4, False), (320, 8, 4, True), (512, 8, 3, True)])
def test_reconstruct_kv_matches_oracle_at_offsets(rank, kv_heads, batch, counted):
    """Rows land at per-sequence starts (after each sequence's raw rows); rows
    past out_rows are skipped, never written.  With per-sequence row counts
    (the latent lengths of a ragged batch, one of them 0) only each
    sequence's first count rows are rebuilt; the rest stay untouched."""
    torch = _cuda()
    from gpu_util import to_bf16
    from slimkv_b200.reconstruct import reconstruct_kv
    rng = np.random.default_rng(rank + batch)
    cap, rows, out_rows, kvd = 300, 257, 340, kv_heads * 128
    lat = oracle.round_bf16(rng.standard_normal((batch, cap, 2 * rank), dtype=np.float32) * 1.3)
    wk = oracle.round_bf16(rng.standard_normal((kvd, rank), dtype=np.float32) * 0.05)
    wv = oracle.round_bf16(rng.standard_normal((kvd, rank), dtype=np.float32) * 0.05)
    bk = oracle.round_bf16(rng.standard_normal(kvd, dtype=np.float32) * 0.1)
    starts = rng.integers(0, out_rows - rows + 1, size=batch).astype(np.int32)
    lat_t = to_bf16(lat)
    key = torch.full((batch, out_rows, kv_heads, 128), float('nan'), dtype=torch.bfloat16, device='cuda')
    value = torch.full_like(key, float('nan'))
    counts = np.full(batch, rows, np.int32)
    if counted:
        counts = rng.integers(1, rows + 1, size=batch).astype(np.int32)
        counts[1] = 0
    reconstruct_kv(lat_t[..., :rank], lat_t[..., rank:], to_bf16(wk), to_bf16(wv), key, value, rows, to_bf16(bk),
                   None, out_start=torch.from_numpy(starts).cuda(),
                   row_count=torch.from_numpy(counts).cuda() if counted else None)
    torch.cuda.synchronize()
    want_k = materialize(lat[:, :rows, :rank], wk, bk).reshape(batch, rows, kv_heads, 128)
    want_v = materialize(lat[:, :rows, rank:], wv, None).reshape(batch, rows, kv_heads, 128)
    k, v = key.float().cpu().numpy(), value.float().cpu().numpy()
    for b in range(batch):
        s, n = int(starts[b]), int(counts[b])
        for got, want in ((k, want_k), (v, want_v)):
            if n:
                assert_near_bits(bf16_bits(got[b, s:s + n]), bf16_bits(want[b, :n]), 5e-3)
            assert np.isnan(got[b, :s]).all() and np.isnan(got[b, s + n:]).all()


@pytest.mark.gpu
@pytest.mark.parametrize('heads,rank,length', [(32, 320, 1), (32, 320, 2), (40, 512, 2), (40, 512, 1)])
def test_reconstruct_decode_matches_oracle(heads, rank, length):
    """The backend's attention rows against the reconstruct oracle, ragged
    lengths and mixed query counts (a Beacon inserted in some rows only)."""
    torch = _cuda()
    from gpu_util import assert_attention_close, to_bf16
    from slimkv_b200 import kernels
    from slimkv_b200.reconstruct import ReconstructDecode
    cos, sin = oracle.rope_tables(128, LLAMA8B['theta'], 16384, LLAMA8B['scaling'])
    cos_t, sin_t = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    c = decode_case(rank + heads + length, batch=3, length=length, history=600, tail=300, heads=heads, rk=rank,
                    rv=rank, bias=True, ragged=True)
    query_len = np.array([length, 1, length])
    c['n_lat'] = c['n_lat'] - (query_len != length)
    B, L, H, D = c['q'].shape
    Hkv = c['kv_heads']
    raw_cap, lat_cap = int(c['n_raw'].max()) + 5, int(c['n_lat'].max()) + 5
    raw_k = np.zeros((B, raw_cap, Hkv, D), np.float32)
    raw_v = np.zeros_like(raw_k)
    for b in range(B):
        n = int(c['n_raw'][b])
        raw_k[b, :n] = oracle.rope_bf16(c['raw_k'][b, :n], cos, sin, c['kpos'][b, :n, None])
        raw_v[b, :n] = c['raw_v'][b, :n]
    lat = np.zeros((B, lat_cap, 2 * rank), np.float32)
    lat[:, :c['lat_k'].shape[1], :rank] = c['lat_k']
    lat[:, :c['lat_v'].shape[1], rank:] = c['lat_v']
    lat_t = to_bf16(lat)
    q_rot = to_bf16(np.stack([oracle.rope_bf16(c['q'][b], cos, sin, c['qpos'][b][:, None]) for b in range(B)]))
    i32 = lambda x: torch.tensor(np.asarray(x), dtype=torch.int32, device='cuda')
    key_full = torch.zeros(B, raw_cap + lat_cap, Hkv, D, dtype=torch.bfloat16, device='cuda')
    rd = ReconstructDecode(raw_k_rot=to_bf16(raw_k), raw_v=to_bf16(raw_v), lat_k=lat_t[..., :rank],
                           lat_v=lat_t[..., rank:], w_k_up=to_bf16(c['uk']), w_v_up=to_bf16(c['uv']),
                           b_k_up=to_bf16(c['bk']), b_v_up=to_bf16(c['bv']), raw_len=i32(c['n_raw']),
                           latent_len=i32(c['n_lat']), query_len=i32(query_len), key_full=key_full,
                           value_full=torch.zeros_like(key_full))
    out = torch.zeros(B, L, H, D, dtype=torch.bfloat16, device='cuda')
    rd(q_rot, out)
    torch.cuda.synchronize()
    for b in range(B):
        l, nr, nl = int(query_len[b]), int(c['n_raw'][b]), int(c['n_lat'][b])
        want = reconstruct_decode_attention(c['q'][b:b + 1, :l], c['raw_k'][b:b + 1, :nr], c['raw_v'][b:b + 1, :nr],
                                            c['lat_k'][b:b + 1, :nl], c['lat_v'][b:b + 1, :nl], c['uk'], c['uv'],
                                            cos, sin, c['qpos'][b:b + 1, :l], c['kpos'][b:b + 1, :nr], l - 1,
                                            uk_bias=c['bk'], uv_bias=c['bv'])
        assert_attention_close(out[b:b + 1, :l].reshape(1, l, H * D), want['out'])
