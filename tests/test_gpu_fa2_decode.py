"""The reference's ``fa2_decode.decode`` contract on the fused sm_100a decode.

``slimkv_b200.fa2_decode.decode`` takes the reference's arguments (an
attention module, hidden states, positions and the reference-layout cache)
and returns what the reference's ``decode`` returns
(slimkv/llama3/fa2_decode.py:77-166).  Inputs are the golden cases that
``tests/golden/make_golden.py`` ran through the reference itself
(``reference_golden.npz``): BASELINE config 1 (one Llama-3.1-8B layer, 2048
latents), an insertion step, a biased 32-head case and the Qwen2.5-14B
geometry (40 heads, rank 512, biases).

Two bars, as ``BASELINE.json`` states them:

* attention output (before ``o_proj``) in the fused op's fp32 output mode
  against the oracle evaluated on the very bf16 inputs the kernel received
  (the module's own bf16 projections): norm-wise relative error <= 2e-3;
* the bf16 output of ``decode`` (after ``o_proj``) against the reference's own
  fp32 result on the unrounded weights: <= 2e-2 absolute.
"""
import numpy as np
import pytest
import torch

from gpu_util import REL_FP32, assert_attention_close

GOLDEN = 'tests/golden/reference_golden.npz'
CASES = {
    'c1': dict(),
    'c1q2': dict(length=2, history=1024, tail=7),
    'bias32': dict(batch=2, length=2, history=300, tail=11, bias=True, seed_w=7, seed_h=8),
    'qwen': dict(batch=1, length=2, history=200, tail=5, rank=512, hidden=5120, heads=40, kv_heads=8, bias=True,
                 seed_w=9, seed_h=10),
}


def _oracle_inputs(attn, case, pk, pv, hidden, positions):
    """The fused op's inputs, recomputed with the module's own (deterministic)
    bf16 projections, as float64-ready numpy arrays for the oracle."""
    B, L = hidden.shape[:2]
    size = L - 1
    f = lambda t: t.detach().float().cpu().numpy()
    with torch.no_grad():
        q = attn.q_proj(hidden)
        if size:
            q = torch.cat([q[:, :1], attn.beacon_q_proj(hidden[:, 1:])], dim=1)
        new_k = attn.k_proj(hidden[:, :1]).reshape(B, 1, attn.num_key_value_heads, attn.head_dim)
        new_v = attn.v_proj(hidden[:, :1]).reshape(B, 1, attn.num_key_value_heads, attn.head_dim)
        raw_k = torch.cat([x.transpose(1, 2) for x in (pk.sink, pk.raw) if x is not None] + [new_k], dim=1)
        raw_v = torch.cat([x.transpose(1, 2) for x in (pv.sink, pv.raw) if x is not None] + [new_v], dim=1)
        lk = [x[:, 0] for x in (pk.history, pk.window) if x is not None]
        lv = [x[:, 0] for x in (pv.history, pv.window) if x is not None]
        if size:
            lk.append(attn.beacon_k_down_proj(hidden[:, 1:]))
            lv.append(attn.beacon_v_down_proj(hidden[:, 1:]))
    S, T, N = case['sink'], case['tail'], case['history']
    idx = np.arange(T) + np.arange(T) // 4
    current = int(positions[0, -L])
    kpos = np.concatenate([np.arange(S), idx + S + N, [current]])[None].repeat(B, 0)
    qpos = positions[:, -L:].cpu().numpy()
    up = lambda m: (f(m.weight), None if m.bias is None else f(m.bias))
    (uk, bk), (uv, bv) = up(attn.beacon_k_up_proj), up(attn.beacon_v_up_proj)
    return dict(q=f(q.reshape(B, L, attn.num_heads, attn.head_dim)), raw_k=f(raw_k), raw_v=f(raw_v),
                lat_k=f(torch.cat(lk, 1)), lat_v=f(torch.cat(lv, 1)), uk=uk, uv=uv, bk=bk, bv=bv, qpos=qpos,
                kpos=kpos, size=size)


@pytest.mark.gpu
@pytest.mark.parametrize('name', list(CASES))
def test_decode_contract_matches_reference(name):
    from cases import config1_layer
    from decode_module import Attention, cache_pair
    from oracle.decode import latent_decode_attention
    from slimkv_b200 import _lib, fa2_decode
    dev = torch.device('cuda', 0)
    golden = np.load(GOLDEN)
    case = config1_layer(**CASES[name])
    attn = Attention(case, dev)
    pk, pv, size, roles = cache_pair(case, dev)
    B, L = case['batch'], case['length']
    hidden = torch.from_numpy(case['hidden']).to(dev, torch.bfloat16)
    past = case['sink'] + case['history'] + case['tail'] + case['win_k'].shape[1]
    positions = torch.arange(past + L, device=dev)[None].expand(B, -1)
    _lib.device_status(clear=True)

    with torch.inference_mode():
        final, none, update = fa2_decode.decode(attn, hidden, positions, (pk, pv, size, roles))
        attn32, _ = fa2_decode.decode_attention(attn, hidden, positions, (pk, pv, size, roles),
                                                out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    # The reference's return contract.
    assert none is None and len(update) == 4 and update[2] == size and update[3] is roles
    assert final.dtype == torch.bfloat16 and final.shape == (B, L, case['hidden_size'])
    assert update[0].shape == (B, case['kv_heads'], 1, case['head_dim']) and update[1].shape == update[0].shape
    if size:
        assert update.key_latents.shape == (B, 1, 1, case['rank'])
        new_lat = golden[f'{name}_new_lat_k']
        assert np.abs(update.key_latents.float().cpu().numpy() - new_lat).max() <= 2e-2
    else:
        assert update.key_latents is None and update.value_latents is None

    # Attention before o_proj, fp32 output mode, vs the oracle on the same inputs.
    x = _oracle_inputs(attn, case, pk, pv, hidden, positions)
    cos, sin = attn.rotary_emb.cos_cached.cpu().numpy(), attn.rotary_emb.sin_cached.cpu().numpy()
    ref = latent_decode_attention(x['q'], x['raw_k'], x['raw_v'], x['lat_k'], x['lat_v'], x['uk'], x['uv'], cos, sin,
                                  x['qpos'], x['kpos'], x['size'], uk_bias=x['bk'], uv_bias=x['bv'])['out']
    err = assert_attention_close(attn32, ref, rel=REL_FP32)

    # decode()'s bf16 output vs the reference's fp32 golden (unrounded weights).
    want = golden[f'{name}_final']
    got = final.float().cpu().numpy()
    abs_err = np.abs(got - want).max()
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert abs_err <= 2e-2, f'{name}: max |final - reference| = {abs_err:.3e}'
    assert rel <= 2e-2, f'{name}: norm-wise relative error vs the reference {rel:.3e}'
    print(f'{name}: attention rel err {err:.2e} (oracle, same inputs); final max abs {abs_err:.2e}, rel {rel:.2e}')
