"""Prefill attention over a latent history (``slimkv_prefill_attention``).

The kernel alone against a PyTorch fp32 attention of the same bf16 inputs:
the chunk part (causal, bottom-right, GQA groups of 4 and 5, a prefix) and
the history part (the absorbed rows of every head against one latent head,
ragged latent counts, non-causal); NaN in every cache row past a length.
The whole chunk attention (absorbed history + causal chunk, LSE-merged, and
the materialised recipe) against the float64 oracle and the reference's own
join (``tests/golden/prefill_attention_golden.npz``).
"""
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from slimkv_b200 import prefill_attention as PA

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).parent / 'golden' / 'prefill_attention_golden.npz')


def torch_attention(q, k, v, kv_len, scale, rpt, causal, offset):
    """fp32 reference: q [B, T, H, dq], k/v [B, cap, Hkv, d]."""
    B, T, H, _ = q.shape
    outs, lses = [], []
    for b in range(B):
        n = int(kv_len[b])
        kb = k[b, :n].float().repeat_interleave(rpt, dim=1)             # [n, H, d]
        vb = v[b, :n].float().repeat_interleave(rpt, dim=1)
        s = torch.einsum('thd,khd->htk', q[b].float(), kb) * scale
        if causal:
            vis = torch.arange(n, device=q.device)[None, :] <= offset + torch.arange(T, device=q.device)[:, None]
            s = s.masked_fill(~vis, float('-inf'))
        lse = torch.logsumexp(s, -1)                                        # [H, T]
        p = torch.exp(s - lse[..., None]).nan_to_num(0.0)
        outs.append(torch.einsum('htk,khd->thd', p, vb))
        lses.append(lse.T)
    return torch.stack(outs), torch.stack(lses)


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize('T,heads,kv_heads,prefix', [(200, 8, 2, 37), (77, 10, 2, 4), (33, 32, 8, 4), (300, 4, 1, 0)])
def test_chunk_part_causal_gqa(T, heads, kv_heads, prefix):
    g = torch.Generator(device='cuda').manual_seed(T + heads)
    B, D, cap = 2, 128, prefix + T + 40
    q = torch.randn(B, T, heads, D, device='cuda', generator=g).to(torch.bfloat16)
    k = torch.full((B, cap, kv_heads, D), float('nan'), device='cuda', dtype=torch.bfloat16)
    v = torch.full_like(k, float('nan'))
    k[:, :prefix + T] = torch.randn(B, prefix + T, kv_heads, D, device='cuda', generator=g).to(torch.bfloat16)
    v[:, :prefix + T] = torch.randn(B, prefix + T, kv_heads, D, device='cuda', generator=g).to(torch.bfloat16)
    kv_len = torch.full((B,), prefix + T, dtype=torch.int32, device='cuda')
    scale = 1 / math.sqrt(D)
    out, lse = PA.attention(q, k, v, kv_len, scale, heads // kv_heads, causal=True, causal_offset=prefix)
    torch.cuda.synchronize()
    want, want_lse = torch_attention(q, k, v, kv_len, scale, heads // kv_heads, True, prefix)
    assert torch.isfinite(out.float()).all()
    assert rel(out, want) < 5e-3
    torch.testing.assert_close(lse, want_lse, atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize('rank,heads', [(320, 32), (160, 40), (256, 8)])
def test_history_part_absorbed_rows(rank, heads):
    """All heads are rows of the one latent head; latent counts 0, 1, 300 and
    129 (a partial last tile), NaN past them."""
    g = torch.Generator(device='cuda').manual_seed(rank + heads)
    lens = [0, 1, 300, 129]
    B, T, cap = len(lens), 21, 340
    q = (torch.randn(B, T, heads, rank, device='cuda', generator=g) * 0.1).to(torch.bfloat16)
    lat = torch.full((B, cap, 2 * rank), float('nan'), device='cuda', dtype=torch.bfloat16)
    for b, n in enumerate(lens):
        lat[b, :n] = torch.randn(n, 2 * rank, device='cuda', generator=g).to(torch.bfloat16)
    k, v = lat[..., :rank].unsqueeze(2), lat[..., rank:].unsqueeze(2)
    kv_len = torch.tensor(lens, dtype=torch.int32, device='cuda')
    scale = 1 / math.sqrt(128)
    out, lse = PA.attention(q, k, v, kv_len, scale, heads)
    torch.cuda.synchronize()
    want, want_lse = torch_attention(q, k, v, kv_len, scale, heads, False, 0)
    assert (out[0] == 0).all() and torch.isinf(lse[0]).all()                # no latents: zero rows, -inf
    assert torch.isfinite(out.float()).all()
    assert rel(out[1:], want[1:]) < 5e-3
    torch.testing.assert_close(lse[1:], want_lse[1:], atol=2e-3, rtol=1e-4)


def golden(name):
    from oracle.bf16 import from_bf16_bits
    g = {k[len(name) + 1:]: v for k, v in GOLDEN.items() if k.startswith(name + '_')}
    t = {}
    for k, v in g.items():
        a = from_bf16_bits(v.view(np.uint16)) if v.dtype == np.int16 else v
        t[k] = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        if v.dtype == np.int16:
            t[k] = t[k].to(torch.bfloat16)
    return t


@pytest.mark.parametrize('name', ['llama_r4', 'qwen_r2'])
def test_chunk_attention_matches_oracle_and_reference_join(name):
    import oracle.prefill_attention as O
    c = golden(name)
    B, T, H, D = c['q'].shape
    n = c['lat_k'].shape[1]
    scale = 1 / math.sqrt(D)
    args = (c['q'], c['sink_k'], c['sink_v'], c['lat_k'], c['lat_v'])
    w = (c['w_k'], c['w_v'], c['cur_k'], c['cur_v'], scale, c.get('b_k'), c.get('b_v'))
    outs = {'materialized': PA.materialized_history_attention(*args, n, *w[:5], uk_bias=w[5], uv_bias=w[6])}
    if c['lat_k'].shape[-1] <= 320:
        lat_len = torch.full((B,), n, dtype=torch.int32, device='cuda')
        outs['absorbed'] = PA.latent_history_attention(*args, lat_len, *w[:5], uk_bias=w[5], uv_bias=w[6])
    torch.cuda.synchronize()
    f = lambda t: None if t is None else t.float().cpu().numpy()
    for b in range(B):
        want, _ = O.prefill_attention(*(f(x[b]) for x in args), *(f(x) for x in w[:2]), f(c['cur_k'][b]),
                                      f(c['cur_v'][b]), scale, f(w[5]), f(w[6]))
        want = torch.from_numpy(want)
        ref = c['out'][b].cpu()
        for kind, o in outs.items():
            got = o[b].float().cpu()
            assert rel(got, want) < 1e-2, (kind, rel(got, want))
            assert rel(got, ref) < 1e-2, (kind, rel(got, ref))
    if 'absorbed' in outs:
        assert rel(outs['absorbed'], outs['materialized']) < 1e-2


def test_prefill_attention_wait_limit_reports_timeout():
    """A wait limit too short for the first copy: the kernel gives up,
    reports SLIMKV_DEVICE_TIMEOUT and the context stays usable."""
    from slimkv_b200 import _lib
    q = torch.randn(1, 64, 4, 128, device='cuda').to(torch.bfloat16)
    k = torch.randn(1, 2048, 1, 128, device='cuda').to(torch.bfloat16)
    kv_len = torch.tensor([2048], dtype=torch.int32, device='cuda')
    _lib.device_status(clear=True)
    PA.attention(q, k, k, kv_len, 0.1, 4, wait_limit_ns=1)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & _lib.DEVICE_TIMEOUT
    out, _ = PA.attention(q, k, k, kv_len, 0.1, 4)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0 and torch.isfinite(out.float()).all()
