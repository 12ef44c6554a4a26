"""Pin the CPU oracle to golden vectors produced by the reference's own code.

The fixture ``tests/golden/reference_golden.npz`` was written by
``tests/golden/make_golden.py`` running the reference SlimKV Python modules
(eager latent decode, rotary, merge, Memory schedule, page IO, split
heuristics) on inputs from ``tests/golden/cases.py``.
"""
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle.decode import latent_decode_attention
from oracle.pages import (BeaconPageLayout, beacon_pages_append, beacon_pages_read,
                          beacon_block_size, raw_page_slots)
from cases import attention_case, config1_layer, LLAMA8B

GOLDEN = np.load(Path(__file__).parent / 'golden' / 'reference_golden.npz')

ATTENTION_SPECS = {
    'latent_q1': (11, 2, 1, 32, 1, 257, 320, 320, False),
    'latent_q2_causal': (12, 2, 2, 32, 1, 130, 160, 192, True),
    'raw_gqa': (13, 3, 1, 32, 8, 37, 128, 128, False),
    'masked_row': (14, 1, 2, 32, 1, 1, 320, 320, True),
    'gqa_q2': (15, 2, 2, 8, 2, 65, 128, 128, True),
}


def assert_lse(actual, expected):
    assert np.array_equal(np.isneginf(actual), np.isneginf(expected))
    finite = np.isfinite(expected)
    np.testing.assert_allclose(actual[finite], expected[finite], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize('name', list(ATTENTION_SPECS))
def test_eager_attention_matches_reference(name):
    c = attention_case(*ATTENTION_SPECS[name], bf16=False)
    out, lse = oracle.eager_attention(c['q'], c['k'], c['v'], c['scale'], c['causal'])
    np.testing.assert_allclose(out, GOLDEN[f'attn_{name}_out'], rtol=1e-5, atol=1e-6)
    assert_lse(lse, GOLDEN[f'attn_{name}_lse'])


def test_masked_row_has_zero_mass_and_neg_inf_lse():
    c = attention_case(*ATTENTION_SPECS['masked_row'], bf16=False)
    out, lse = oracle.eager_attention(c['q'], c['k'], c['v'], c['scale'], True)
    assert np.isneginf(lse[..., 0]).all() and (out[:, 0] == 0).all()


def test_merge_matches_reference():
    rng = np.random.default_rng(21)
    raw = rng.standard_normal((2, 32, 2, 128), dtype=np.float32)
    lat = rng.standard_normal((2, 32, 2, 128), dtype=np.float32)
    rl = rng.standard_normal((2, 32, 2), dtype=np.float32) * 4
    ll = rng.standard_normal((2, 32, 2), dtype=np.float32) * 4
    ll[..., 0] = -np.inf
    merged = oracle.merge_attention(raw, rl, lat, ll)
    np.testing.assert_allclose(merged, GOLDEN['merge_out'], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(merged[..., 0, :], raw[..., 0, :])


def test_rope_tables_are_bit_exact():
    cos, sin = oracle.rope_tables(128, LLAMA8B['theta'], LLAMA8B['max_positions'], LLAMA8B['scaling'])
    rows = GOLDEN['rope_llama3_rows']
    assert np.array_equal(cos[rows].view(np.uint32), GOLDEN['rope_llama3_cos'].view(np.uint32))
    assert np.array_equal(sin[rows].view(np.uint32), GOLDEN['rope_llama3_sin'].view(np.uint32))
    cos, sin = oracle.rope_tables(128, 1e6, 32768)
    assert np.array_equal(cos[rows[:9]].view(np.uint32), GOLDEN['rope_qwen_cos'].view(np.uint32))
    assert np.array_equal(sin[rows[:9]].view(np.uint32), GOLDEN['rope_qwen_sin'].view(np.uint32))


def test_rope_bf16_is_bit_exact():
    cos, sin = oracle.rope_tables(128, LLAMA8B['theta'], LLAMA8B['max_positions'], LLAMA8B['scaling'])
    q = oracle.from_bf16_bits(GOLDEN['rope_q_in'].view(np.uint16))
    k = oracle.from_bf16_bits(GOLDEN['rope_k_in'].view(np.uint16))
    pos = GOLDEN['rope_pos']
    # The reference rotates q at the last Q positions of position_ids.
    qo = oracle.rope_bf16(q, cos, sin, pos[:, None, -q.shape[2]:])
    ko = oracle.rope_bf16(k, cos, sin, pos[:, None, :])
    assert np.array_equal(oracle.bf16_bits(qo), GOLDEN['rope_q_out'].view(np.uint16))
    assert np.array_equal(oracle.bf16_bits(ko), GOLDEN['rope_k_out'].view(np.uint16))


def _layer_inputs(c):
    """Recreate, in numpy, the tensors the reference decode computed from hidden."""
    w = c['weights']
    b, L, H, Hkv, d = c['batch'], c['length'], c['heads'], c['kv_heads'], c['head_dim']
    bias = c['bias']

    def lin(x, name, bname):
        y = x @ w[name].T
        return y + w[bname] if bias and bname else y

    x = c['hidden']
    q = lin(x, 'q_proj', 'q_bias')
    if L == 2:
        q[:, 1:] = lin(x[:, 1:], 'beacon_q_proj', 'beacon_q_bias')
    q = q.reshape(b, L, H, d)
    new_k = lin(x[:, :1], 'k_proj', 'k_bias').reshape(b, 1, Hkv, d)
    new_v = lin(x[:, :1], 'v_proj', 'v_bias').reshape(b, 1, Hkv, d)
    raw_k = np.concatenate([c['sink_k'], c['tail_k'], new_k], axis=1)
    raw_v = np.concatenate([c['sink_v'], c['tail_v'], new_v], axis=1)
    lat_k = np.concatenate([c['hist_k'], c['win_k']], axis=1)
    lat_v = np.concatenate([c['hist_v'], c['win_v']], axis=1)
    if L == 2:
        lat_k = np.concatenate([lat_k, x[:, 1:] @ w['k_down'].T], axis=1)
        lat_v = np.concatenate([lat_v, x[:, 1:] @ w['v_down'].T], axis=1)
    S, N, T = c['sink'], c['history'], c['tail']
    n_win = c['win_k'].shape[1]
    current = S + N + T + n_win
    qpos = np.tile(current + np.arange(L), (b, 1))
    idx = np.arange(T) + np.arange(T) // 4
    kpos = np.tile(oracle.raw_key_positions(S, idx, N, current), (b, 1))
    return q.astype(np.float32), raw_k, raw_v, lat_k, lat_v, qpos, kpos


DECODE_CASES = {
    'c1': dict(),
    'c1q2': dict(length=2, history=1024, tail=7),
    'small_bias': dict(batch=2, length=2, history=40, tail=11, rank=16, hidden=256, heads=8,
                       kv_heads=2, head_dim=32, bias=True, seed_w=5, seed_h=6),
}


@pytest.mark.parametrize('name', list(DECODE_CASES))
def test_latent_decode_matches_reference(name):
    c = config1_layer(**DECODE_CASES[name])
    w = c['weights']
    q, raw_k, raw_v, lat_k, lat_v, qpos, kpos = _layer_inputs(c)
    cos, sin = oracle.rope_tables(c['head_dim'], LLAMA8B['theta'], 65536, LLAMA8B['scaling'])
    r = latent_decode_attention(q, raw_k, raw_v, lat_k, lat_v, w['k_up'], w['v_up'], cos, sin,
                                qpos, kpos, c['length'] - 1,
                                uk_bias=w.get('k_up_bias'), uv_bias=w.get('v_up_bias'), dtype='fp32')
    tol = dict(rtol=2e-4, atol=2e-5)
    np.testing.assert_allclose(r['q_rot'], GOLDEN[f'{name}_q_rot'], **tol)
    np.testing.assert_allclose(r['k_rot'], GOLDEN[f'{name}_k_rot'], **tol)
    np.testing.assert_allclose(r['raw_out'].transpose(0, 2, 1, 3), GOLDEN[f'{name}_raw_out'], **tol)
    assert_lse(r['raw_lse'], GOLDEN[f'{name}_raw_lse'])
    np.testing.assert_allclose(r['q_lat'].transpose(0, 2, 1, 3), GOLDEN[f'{name}_q_lat'], **tol)
    np.testing.assert_allclose(r['latent_branch_out'], GOLDEN[f'{name}_lat_out'], **tol)
    np.testing.assert_allclose(r['latent_branch_lse'], GOLDEN[f'{name}_lat_lse'], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(r['out'], GOLDEN[f'{name}_attn'], **tol)
    final = r['out'] @ w['o_proj'].T + (w['o_bias'] if c['bias'] else 0)
    np.testing.assert_allclose(final, GOLDEN[f'{name}_final'], rtol=5e-4, atol=5e-5)


@pytest.mark.parametrize('tag,window,sink,prefill,steps',
                         [('w8', 8, 1, 17, 44), ('w16s2', 16, 2, 5, 60)])
def test_decode_schedule_matches_reference(tag, window, sink, prefill, steps):
    s = oracle.FastDecodeSchedule(window, 4, sink)
    s.prefill(prefill)
    for i in range(steps):
        rec = s.decode()
        assert rec['size'] == GOLDEN[f'sched_{tag}_sizes'][i], i
        mem = (s.sink, s.history, s.raw + s.win)
        assert tuple(GOLDEN[f'sched_{tag}_mem'][i]) == mem, (i, mem)
        assert s.remainder == GOLDEN[f'sched_{tag}_rem'][i]
        assert bool(s.is_full_window) == bool(GOLDEN[f'sched_{tag}_full'][i])
        roles = GOLDEN[f'sched_{tag}_roles'][i]
        assert np.array_equal(rec['roles'], roles[roles != -9]), i
        raw = GOLDEN[f'sched_{tag}_rawidx'][i]
        expected = raw[raw != -9].astype(np.int64)
        actual = np.zeros(0, np.int64) if s.window_raw_indices is None else s.window_raw_indices
        assert np.array_equal(actual, expected), i


def test_prefill_interleave_matches_reference():
    s = oracle.FastDecodeSchedule(16, 4, 0)
    records = []
    for count in [3, 5, 9, 2, 13, 20, 1, 1, 1]:
        records += s.prefill(count)
    golden = GOLDEN['interleave_roles']
    assert len(records) == len(golden)
    for rec, row in zip(records, golden):
        assert np.array_equal(rec['roles'], row[row != -9])


def test_paged_restore_roles_match_schedule():
    for processed in [0, 1, 3, 4, 5, 191, 192, 1023, 1024, 1025, 4099]:
        roles, raw_idx, hist, beacons = oracle.paged_restore_roles(processed, 1024, 4)
        assert hist == processed // 1024 * 256 and beacons == processed // 4
        s = oracle.FastDecodeSchedule(1024, 4, 1)
        if processed:
            s.prefill(processed)
        if processed % 1024:
            assert np.array_equal(roles, s.roles)
            assert np.array_equal(raw_idx, s.window_raw_indices)


def test_beacon_pages_match_reference_bytes():
    layout = BeaconPageLayout(4, 2, 3, 5, 4)
    backing = np.full((12, layout.page_elements + 7), -13, dtype=np.float32)
    for index, table in enumerate([np.array([7, 2, 9]), np.array([4, 1, 10])]):
        k = np.arange(18, dtype=np.float32).reshape(6, 3) + index * 32
        v = np.arange(30, dtype=np.float32).reshape(6, 5) + index * 32
        beacon_pages_append(backing, table, 0, k[:3], v[:3], layout)
        beacon_pages_append(backing, table, 3, k[3:], v[3:], layout)
        sink = np.full(4, index + 1, dtype=np.float32)
        backing[table[0], :layout.sink_elements] = np.concatenate([sink, sink + 2])
        rk, rv = beacon_pages_read(backing, table, 6, layout)
        assert np.array_equal(rk, k) and np.array_equal(rv, v)
    assert np.array_equal(oracle.bf16_bits(backing), GOLDEN['pages_small'].view(np.uint16))

    layout = BeaconPageLayout(192, 4, 320, 320, 1024)
    assert (layout.slots, layout.storage_rows) == (48, 52)
    k = oracle.from_bf16_bits(GOLDEN['pages_r4_kin'].view(np.uint16))[0, 0]
    v = oracle.from_bf16_bits(GOLDEN['pages_r4_vin'].view(np.uint16))[0, 0]
    flat = np.zeros((9, layout.storage_rows * layout.width), np.float32)
    table = np.array([5, 0, 8, 3, 6])
    beacon_pages_append(flat, table, 0, k[:130], v[:130], layout)
    beacon_pages_append(flat, table, 130, k[130:], v[130:], layout)
    assert np.array_equal(oracle.bf16_bits(flat).reshape(9, 52, 640), GOLDEN['pages_r4'].view(np.uint16))


def test_raw_pages_match_reference_bytes():
    pages = np.zeros((8, 4, 2, 2, 3), np.float32)
    key = np.arange(42, dtype=np.float32).reshape(2, 7, 3)
    block, row = raw_page_slots(np.array([5, 2, 6, 1]), 5, 7, 4)
    for i in range(7):
        pages[block[i], row[i], 0] = key[:, i]
        pages[block[i], row[i], 1] = -key[:, i]
    assert np.array_equal(oracle.bf16_bits(pages), GOLDEN['raw_pages'].view(np.uint16))


def test_vllm_page_geometry_known_answers():
    # r4/t4: page of 16 raw tokens x K,V x 1024 x 2 bytes = 64 KiB holds 48
    # slots of 640 after the 2048-element sink; r8/t8: 96 slots of 320.
    assert beacon_block_size(4, 1024, 640) == 192
    assert beacon_block_size(8, 1024, 320) == 768
    assert BeaconPageLayout(192, 4, 320, 320, 1024).page_elements == 32768
    assert BeaconPageLayout(768, 8, 160, 160, 1024).page_elements == 32768


def test_split_heuristics_match_reference():
    for width, keys, heads, sms, expected in GOLDEN['splits']:
        assert oracle.original_splits(int(width), int(keys), int(heads), int(sms)) == expected
    for length in [8256, 16448, 32832]:
        assert oracle.original_splits(320, length, 32, 78) == 3
        assert oracle.original_splits(256, length, 32, 78) == 9
