"""Pin the numpy decode-layer restatement (``oracle/cpu_decode.py``) to the
reference's own ``fa2_decode.decode`` outputs.

``tests/golden/make_golden.py`` (``gen_decode``) ran the reference's eager
decode (slimkv/llama3/fa2_decode.py:77-166 with latent_decode.py:16-41) on
the ``config1_layer`` cases and stored its fp32 result after ``o_proj``
(``{case}_final``) and the new Beacon latents.  ``CpuDecodeLayer.attend``
gets the same weights, caches (pre-RoPE sink and raw keys, history and
open-window latents) and attention inputs, with Llama-3-scaled RoPE tables,
and must agree to fp32 rounding: BASELINE config 1 (2048 latents), an
insertion step, a biased 32-head case and the Qwen2.5-14B geometry.
"""
from pathlib import Path

import numpy as np
import pytest

from cases import LLAMA8B, config1_layer
from oracle.cpu_decode import CpuDecodeLayer
from oracle.rope import rope_tables

GOLDEN = np.load(Path(__file__).parent / 'golden' / 'reference_golden.npz')
CASES = {
    'c1': dict(),
    'c1q2': dict(length=2, history=1024, tail=7),
    'bias32': dict(batch=2, length=2, history=300, tail=11, bias=True, seed_w=7, seed_h=8),
    'qwen': dict(batch=1, length=2, history=200, tail=5, rank=512, hidden=5120, heads=40, kv_heads=8, bias=True,
                 seed_w=9, seed_h=10),
}


def _layer(case):
    B, S, T, N = case['batch'], case['sink'], case['tail'], case['history']
    n_win = case['win_k'].shape[1]
    idx = np.arange(T) + np.arange(T) // 4
    seqs = [dict(sink_k=case['sink_k'][b], sink_v=case['sink_v'][b], raw_k=case['tail_k'][b],
                 raw_v=case['tail_v'][b], raw_pos=idx + S + N,
                 lat_k=np.concatenate([case['hist_k'][b], case['win_k'][b]]),
                 lat_v=np.concatenate([case['hist_v'][b], case['win_v'][b]]), position=S + N + T + n_win)
            for b in range(B)]
    cos, sin = rope_tables(case['head_dim'], LLAMA8B['theta'], S + N + T + n_win + 4, LLAMA8B['scaling'])
    return CpuDecodeLayer(case['weights'], seqs, case['heads'], case['kv_heads'], case['head_dim'], cos, sin)


@pytest.mark.parametrize('name', list(CASES))
def test_port_matches_reference_decode(name):
    case = config1_layer(**CASES[name])
    B, L = case['batch'], case['length']
    h = np.zeros((B, 2, case['hidden_size']), np.float32)
    h[:, :L] = case['hidden']
    out, lat_k, _ = _layer(case).attend(h, [L] * B)
    want = GOLDEN[f'{name}_final']
    got = out[:, :L]
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 1e-5, f'{name}: norm-wise relative error {rel:.2e}'
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)
    if L == 2:
        np.testing.assert_allclose(lat_k, GOLDEN[f'{name}_new_lat_k'][:, 0, 0], rtol=1e-4, atol=1e-5)


def test_rope_scaling_changes_the_answer():
    """The reference's Llama-3 RoPE scaling matters at these positions: the
    port with unscaled tables misses the golden output."""
    case = config1_layer()
    layer = _layer(case)
    pos = layer.seqs[0]['position'] + 4
    layer.cos, layer.sin = rope_tables(case['head_dim'], LLAMA8B['theta'], pos, None)
    h = np.zeros((1, 2, case['hidden_size']), np.float32)
    h[:, :1] = case['hidden']
    out, _, _ = layer.attend(h, [1])
    want = GOLDEN['c1_final']
    assert np.linalg.norm(out[:, :1] - want) / np.linalg.norm(want) > 1e-3
