"""Generate golden vectors by running the reference SlimKV Python code.

Usage (needs a checkout of the reference; it is not shipped with this repo)::

    python tests/golden/make_golden.py --reference <path to SlimKV checkout>

The reference imports two optional packages at module load that its hot path
never uses; minimal stand-ins for them (``pytz`` with a version string and
``accelerate.Accelerator``) are created in a temporary directory.  Inputs come
from ``tests/golden/cases.py`` (numpy ``default_rng``), are handed to the
reference as torch CPU tensors, and the reference's outputs are stored as
compressed ``.npz`` fixtures next to this script.  Nothing here is used at
run time by the library.
"""
import argparse
import math
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _stubs():
    d = Path(tempfile.mkdtemp(prefix='slimkv_stubs_'))
    (d / 'pytz').mkdir()
    (d / 'pytz' / '__init__.py').write_text('__version__ = "2024.1"\n')
    (d / 'accelerate').mkdir()
    (d / 'accelerate' / '__init__.py').write_text('__version__ = "1.0.0"\nclass Accelerator:\n    pass\n')
    return d


def _t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x))


def gen_attention(out):
    import torch
    from slimkv.llama3.latent_decode import eager_forward
    from cases import attention_case
    specs = {
        'latent_q1': (11, 2, 1, 32, 1, 257, 320, 320, False),
        'latent_q2_causal': (12, 2, 2, 32, 1, 130, 160, 192, True),
        'raw_gqa': (13, 3, 1, 32, 8, 37, 128, 128, False),
        'masked_row': (14, 1, 2, 32, 1, 1, 320, 320, True),
        'gqa_q2': (15, 2, 2, 8, 2, 65, 128, 128, True),
    }
    for name, spec in specs.items():
        c = attention_case(*spec, bf16=False)
        o, lse = eager_forward(_t(c['q']), _t(c['k']), _t(c['v']), c['scale'], c['causal'])
        out[f'attn_{name}_out'] = o.numpy()
        out[f'attn_{name}_lse'] = lse.numpy()


def gen_merge(out):
    from slimkv.llama3.fa2_decode import merge_attention
    rng = np.random.default_rng(21)
    raw = rng.standard_normal((2, 32, 2, 128), dtype=np.float32)
    lat = rng.standard_normal((2, 32, 2, 128), dtype=np.float32)
    rl = rng.standard_normal((2, 32, 2), dtype=np.float32) * 4
    ll = rng.standard_normal((2, 32, 2), dtype=np.float32) * 4
    ll[..., 0] = -np.inf
    out['merge_out'] = merge_attention(_t(raw), _t(rl), _t(lat), _t(ll)).numpy()


def gen_rope(out):
    import torch
    from slimkv.modeling_utils import get_rope
    from cases import LLAMA8B
    sc = dict(LLAMA8B['scaling'], type='llama3')
    rope = get_rope(128, LLAMA8B["theta"], 131072, sc)
    rows = np.array([0, 1, 2, 3, 4, 1000, 8191, 8192, 32767, 40000, 65535, 131071])
    out['rope_llama3_rows'] = rows
    out['rope_llama3_cos'] = rope.cos_cached[rows].numpy()
    out['rope_llama3_sin'] = rope.sin_cached[rows].numpy()
    qwen = get_rope(128, 1e6, 32768, None)
    out['rope_qwen_cos'] = qwen.cos_cached[rows[:9]].numpy()
    out['rope_qwen_sin'] = qwen.sin_cached[rows[:9]].numpy()
    rng = np.random.default_rng(31)
    q = torch.from_numpy(rng.standard_normal((2, 32, 2, 128), dtype=np.float32) * 2).to(torch.bfloat16)
    k = torch.from_numpy(rng.standard_normal((2, 8, 70, 128), dtype=np.float32) * 2).to(torch.bfloat16)
    pos = torch.from_numpy(rng.integers(0, 131072, size=(2, 70)))
    qo, ko = rope(q, k, pos)                     # bf16 rotary of the reference
    out['rope_q_in'] = q.view(torch.int16).numpy()
    out['rope_k_in'] = k.view(torch.int16).numpy()
    out['rope_pos'] = pos.numpy()
    out['rope_q_out'] = qo.view(torch.int16).numpy()
    out['rope_k_out'] = ko.view(torch.int16).numpy()


def _attention_module(layer):
    import torch
    from slimkv.llama3.configuration_llama import LlamaConfig
    from slimkv.llama3.modeling_llama import LlamaAttention
    from cases import LLAMA8B
    c = layer
    config = LlamaConfig(
        vocab_size=128, hidden_size=c['hidden_size'], intermediate_size=64,
        num_hidden_layers=1, num_attention_heads=c['heads'], num_key_value_heads=c['kv_heads'],
        max_position_embeddings=8192, rope_theta=LLAMA8B['theta'],
        rope_scaling=dict(LLAMA8B['scaling'], rope_type='llama3'),
        attention_bias=c['bias'], beacon_param=['q', 'k', 'v'], beacon_window=1024,
        beacon_stride=1024, beacon_ratio=[4], beacon_ratio_mix='sequence',
        beacon_sink_size=c['sink'], beacon_skip_rope_for_beacon_k=True,
        beacon_k_compression='lowrank_svd', beacon_v_compression='lowrank_svd',
        beacon_k_latent_head_dim_list=[c['rank'] // c['kv_heads']],
        beacon_v_latent_head_dim_list=[c['rank'] // c['kv_heads']],
        beacon_decode_backend='latent', torch_dtype=torch.float32)
    config._attn_implementation = 'eager'
    attn = LlamaAttention(config, layer_idx=0).eval()
    w = c['weights']
    pairs = [('q_proj', attn.q_proj, 'q_bias'), ('k_proj', attn.k_proj, 'k_bias'),
             ('v_proj', attn.v_proj, 'v_bias'), ('o_proj', attn.o_proj, 'o_bias'),
             ('beacon_q_proj', attn.beacon_q_proj, 'beacon_q_bias'),
             ('k_down', attn.beacon_k_down_proj, None), ('k_up', attn.beacon_k_up_proj, 'k_up_bias'),
             ('v_down', attn.beacon_v_down_proj, None), ('v_up', attn.beacon_v_up_proj, 'v_up_bias')]
    with torch.no_grad():
        for name, mod, bname in pairs:
            mod.weight.copy_(_t(w[name]))
            if mod.bias is not None:
                mod.bias.copy_(_t(w[bname]))
    return attn


def gen_decode(out, name, layer):
    """Run ``fa2_decode.decode`` with the eager backend and record every stage."""
    import torch
    from slimkv.llama3 import fa2_decode
    from slimkv.llama3.latent_decode import eager_forward
    from slimkv.llama3.memory import ReconstructionCache
    c = layer
    attn = _attention_module(c)
    b, L, S, T, N = c['batch'], c['length'], c['sink'], c['tail'], c['history']
    size = L - 1

    def bhsd(x):
        return None if x is None or x.shape[1] == 0 else _t(x).transpose(1, 2).contiguous()

    def lat(x):
        return None if x.shape[1] == 0 else _t(x)[:, None].contiguous()

    raw_idx = torch.arange(T) + torch.arange(T) // 4 if T else None
    n_win = c['win_k'].shape[1]
    roles = torch.zeros(T + n_win + 1 + size, dtype=torch.long)
    if T:
        roles[:T + n_win] = 0
        roles[4::5] = 1
    if size:
        roles[-1] = 1
    window_roles = (roles[:T + n_win] != 0) if (T + n_win) else None
    pk = ReconstructionCache(bhsd(c['sink_k']), lat(c['hist_k']), bhsd(c['tail_k']), lat(c['win_k']),
                             window_roles, c['kv_heads'], c['head_dim'], 'k', raw_idx)
    pv = ReconstructionCache(bhsd(c['sink_v']), lat(c['hist_v']), bhsd(c['tail_v']), lat(c['win_v']),
                             window_roles, c['kv_heads'], c['head_dim'], 'v', raw_idx)
    past_len = S + N + T + n_win
    positions = torch.arange(past_len + L)[None].expand(b, -1)
    calls = []

    def recording(q, k, v, scale, causal=False):
        o, lse = eager_forward(q, k, v, scale, causal)
        calls.append((q.numpy().copy(), k.numpy().copy(), o.numpy().copy(), lse.numpy().copy()))
        return o, lse

    captured = {}
    original = attn.o_proj_with_beacon

    def capture(x, s, i):
        captured['x'] = x.detach().numpy().copy()
        return original(x, s, i)

    attn.o_proj_with_beacon = capture
    with torch.inference_mode():
        result, _, update = fa2_decode.decode(attn, _t(c['hidden']), positions,
                                              (pk, pv, size, roles), forward=recording)
    out[f'{name}_q_rot'] = calls[0][0]
    out[f'{name}_k_rot'] = calls[0][1]
    out[f'{name}_raw_out'] = calls[0][2]
    out[f'{name}_raw_lse'] = calls[0][3]
    out[f'{name}_q_lat'] = calls[1][0]
    out[f'{name}_lat_out'] = calls[1][2]
    out[f'{name}_lat_lse'] = calls[1][3]
    out[f'{name}_attn'] = captured['x']
    out[f'{name}_final'] = result.numpy()
    if size:
        out[f'{name}_new_lat_k'] = update.key_latents.numpy()


def gen_schedule(out, ref_tests):
    """Record fast-decode metadata of a real reference model across windows."""
    import torch
    from unittest.mock import patch
    sys.path.insert(0, str(ref_tests))
    from test_llama_reconstruction_cache import make_model
    from test_llama_fa2_decode import reference_forward
    for tag, kwargs, prefill, steps in [
            ('w8', {}, 17, 44),
            ('w16s2', dict(beacon_window=16, beacon_stride=16, beacon_sink_size=2), 5, 60)]:
        torch.manual_seed(42)
        model = make_model(beacon_decode_backend='fa2', **kwargs)
        sizes, roles, raw_idx, mem, rem, full = [], [], [], [], [], []
        with torch.inference_mode(), patch('slimkv.llama3.fa2_decode.flash_forward',
                                           side_effect=reference_forward):
            model(input_ids=torch.arange(prefill)[None] % 64)
            for i in range(steps):
                model(input_ids=torch.tensor([[(prefill + 1 + i) % 64]]))
                m = model.memory
                sizes.append(m._all_beacon_sizes[-1])
                roles.append(m._beacon_indices.tolist())
                raw_idx.append([] if m._window_raw_indices is None else m._window_raw_indices.tolist())
                mem.append(list(m.get_memory_size()))
                rem.append(m._interleave_remainder)
                full.append(bool(m._is_full_window))
        out[f'sched_{tag}_sizes'] = np.array(sizes)
        out[f'sched_{tag}_mem'] = np.array(mem)
        out[f'sched_{tag}_rem'] = np.array(rem)
        out[f'sched_{tag}_full'] = np.array(full)
        out[f'sched_{tag}_roles'] = np.array([np.pad(r, (0, 64 - len(r)), constant_values=-9) for r in roles])
        out[f'sched_{tag}_rawidx'] = np.array([np.pad(r, (0, 64 - len(r)), constant_values=-9) for r in raw_idx])


def gen_model_decode(out, ref_tests):
    """Prefill + decode of the reference's SlimKV Llama (``TINY_MODEL``).

    The reference model (fast latent decode, ``beacon_decode_backend='fa2'``,
    with the reference test suite's fp32 ``reference_forward`` standing in for
    the FA2 kernel as its own tests do) prefills ``prefill`` tokens, and its
    memory after prefill is recorded per layer (sinks, Beacon latents of the
    completed windows, raw tail and window latents of the open window); then
    ``steps`` single-token decode calls record fp32 logits.  The window is 64
    tokens, so the decode crosses one window rollover and inserts a Beacon
    every fourth step.
    """
    import torch
    from unittest.mock import patch
    sys.path.insert(0, str(ref_tests))
    from test_llama_fa2_decode import reference_forward
    from slimkv.llama3.configuration_llama import LlamaConfig
    from slimkv.llama3.memory import LlamaMemory
    from slimkv.llama3.modeling_llama import LlamaForCausalLM
    from cases import LLAMA8B, TINY_MODEL, tiny_model_tokens, tiny_model_weights
    s = TINY_MODEL
    config = LlamaConfig(
        vocab_size=s['vocab'], hidden_size=s['hidden'], intermediate_size=s['intermediate'],
        num_hidden_layers=s['layers'], num_attention_heads=s['heads'], num_key_value_heads=s['kv_heads'],
        max_position_embeddings=8192, rope_theta=s['theta'], rms_norm_eps=s['rms_eps'],
        rope_scaling=dict(LLAMA8B['scaling'], rope_type='llama3'), beacon_param=['q', 'k', 'v'],
        beacon_window=s['window'], beacon_stride=s['window'], beacon_ratio=[s['ratio']],
        beacon_ratio_mix='sequence', beacon_sink_size=s['sink'], beacon_skip_rope_for_beacon_k=True,
        beacon_k_compression='lowrank_svd', beacon_v_compression='lowrank_svd',
        beacon_k_latent_head_dim_list=[s['rank'] // s['kv_heads']] * s['layers'],
        beacon_v_latent_head_dim_list=[s['rank'] // s['kv_heads']] * s['layers'],
        beacon_decode_backend='fa2', torch_dtype=torch.float32)
    config._attn_implementation = 'eager'
    model = LlamaForCausalLM(config)
    model.memory = LlamaMemory(config)
    weights = tiny_model_weights()
    params = dict(model.named_parameters())
    assert set(params) == set(weights), sorted(set(params) ^ set(weights))
    with torch.no_grad():
        for name, p in params.items():
            p.copy_(_t(weights[name]))
    model.eval()
    prefill, steps = tiny_model_tokens()
    logits = []
    with torch.inference_mode(), patch('slimkv.llama3.fa2_decode.flash_forward', side_effect=reference_forward):
        model(input_ids=_t(prefill)[None])
        m = model.memory
        for i in range(s['layers']):
            (sk, sv), (hk, hv) = m.sink_activations[i], m.beacon_activations[i]
            (rk, rv), (wk, wv) = m.raw_activations[i], m.window_beacon_activations[i]
            out[f'model_l{i}_sink_k'], out[f'model_l{i}_sink_v'] = sk[0].numpy(), sv[0].numpy()
            out[f'model_l{i}_hist_k'], out[f'model_l{i}_hist_v'] = hk[0, 0].numpy(), hv[0, 0].numpy()
            out[f'model_l{i}_raw_k'], out[f'model_l{i}_raw_v'] = rk[0].numpy(), rv[0].numpy()
            out[f'model_l{i}_win_k'], out[f'model_l{i}_win_v'] = wk[0, 0].numpy(), wv[0, 0].numpy()
        out['model_window_raw_indices'] = m._window_raw_indices.numpy()
        out['model_remainder'] = np.array(m._interleave_remainder)
        for tok in steps:
            logits.append(model(input_ids=torch.tensor([[int(tok)]])).logits[0, -1].float().numpy())
    out['model_logits'] = np.stack(logits)


def gen_interleave(out):
    """Prefill interleave roles from the reference ``Memory._step``."""
    import torch
    from slimkv.llama3.configuration_llama import LlamaConfig
    from slimkv.memory import Memory
    config = LlamaConfig(vocab_size=64, hidden_size=32, intermediate_size=48, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, beacon_window=16,
                         beacon_stride=16, beacon_ratio=[4], beacon_ratio_mix='sequence',
                         beacon_sink_size=0, beacon_param=['k', 'v'], torch_dtype=torch.float32)
    config._attn_implementation = 'eager'
    records = []
    mem = Memory(config)
    mem.eval()
    mem.reset()
    for count in [3, 5, 9, 2, 13, 20, 1, 1, 1]:
        mem.prepare(torch.zeros(1, count, dtype=torch.long), None, None)
        while not mem.finish:
            ids, mask, pos, past, labels = mem.step()
            records.append(list(past[0][3].tolist()))
            # Emulate update_memory's length effect with empty caches.
            mem.update_memory([(None, None, past[0][2], past[0][3])])
    out['interleave_roles'] = np.array([np.pad(r, (0, 40 - len(r)), constant_values=-9) for r in records])


def gen_pages(out):
    import torch
    from slimkv.vllm_plugin.paged_cache import BeaconPageLayout, BeaconPages, RawPages
    layout = BeaconPageLayout(4, 2, 3, 5, 4)
    backing = torch.full((12, layout.page_elements + 7), -13, dtype=torch.bfloat16)
    pages = BeaconPages(backing[:, :layout.page_elements], layout)
    for index, table in enumerate([torch.tensor([7, 2, 9]), torch.tensor([4, 1, 10])]):
        k = torch.arange(18).reshape(1, 1, 6, 3).to(torch.bfloat16) + index * 32
        v = torch.arange(30).reshape(1, 1, 6, 5).to(torch.bfloat16) + index * 32
        pages.append(table, 0, k[:, :, :3], v[:, :, :3])
        pages.append(table, 3, k[:, :, 3:], v[:, :, 3:])
        sink = torch.full((1, 1, 1, 4), index + 1, dtype=torch.bfloat16)
        pages.write_sink(table[0], sink, sink + 2)
    out['pages_small'] = backing.view(torch.int16).numpy()
    # Production r4/t4 layout: 192 raw tokens per page, 48 slots of 640.
    layout = BeaconPageLayout(192, 4, 320, 320, 1024)
    rng = np.random.default_rng(41)
    backing = torch.zeros((9, layout.storage_rows, layout.width), dtype=torch.bfloat16)
    pages = BeaconPages(backing, layout)
    table = torch.tensor([5, 0, 8, 3, 6])
    k = torch.from_numpy(rng.standard_normal((1, 1, 200, 320), dtype=np.float32)).to(torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((1, 1, 200, 320), dtype=np.float32)).to(torch.bfloat16)
    pages.append(table, 0, k[:, :, :130], v[:, :, :130])
    pages.append(table, 130, k[:, :, 130:], v[:, :, 130:])
    out['pages_r4_kin'] = k.view(torch.int16).numpy()
    out['pages_r4_vin'] = v.view(torch.int16).numpy()
    out['pages_r4'] = backing.view(torch.int16).numpy()
    raw = RawPages(torch.zeros(8, 4, 2, 2, 3, dtype=torch.bfloat16))
    key = torch.arange(42).reshape(1, 2, 7, 3).to(torch.bfloat16)
    raw.write(torch.tensor([5, 2, 6, 1]), 5, key, -key)
    out['raw_pages'] = raw.pages.view(torch.int16).numpy()


def _prefill_module(seed):
    """A small bf16 Llama attention with low-rank Beacon K/V (R_k 16, R_v 32)."""
    import torch
    from slimkv.llama3.configuration_llama import LlamaConfig
    from slimkv.llama3.modeling_llama import LlamaAttention
    from cases import LLAMA8B
    config = LlamaConfig(
        vocab_size=64, hidden_size=128, intermediate_size=64, num_hidden_layers=1,
        num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
        rope_theta=LLAMA8B['theta'], rope_scaling=dict(LLAMA8B['scaling'], rope_type='llama3'),
        attention_bias=True, beacon_param=['q', 'k', 'v'], beacon_window=16, beacon_stride=16,
        beacon_ratio=[4], beacon_ratio_mix='sequence', beacon_sink_size=1,
        beacon_skip_rope_for_beacon_k=True, beacon_k_compression='lowrank_svd',
        beacon_v_compression='lowrank_svd', beacon_k_latent_head_dim_list=[8],
        beacon_v_latent_head_dim_list=[16], beacon_decode_backend='latent', torch_dtype=torch.float32)
    config._attn_implementation = 'eager'
    torch.manual_seed(seed)
    attn = LlamaAttention(config, layer_idx=0).eval()
    with torch.no_grad():
        for p in attn.parameters():
            p.normal_(0, 0.1)
    # The fp32 rotary tables as built (the bf16 cast below rounds them).
    tables = attn.rotary_emb.cos_cached[:512].clone(), attn.rotary_emb.sin_cached[:512].clone()
    return attn.to(torch.bfloat16), tables


def gen_prefill(out):
    """Role-selected projections, latent packing and prefill RoPE of the reference.

    ``qkv_proj_with_beacon`` + ``_incremental_cache`` run under prefill
    metadata (``prepare_metadata``'s index lists) on a bf16 module; the
    prefill RoPE comes from ``_apply_rotary_with_beacon`` (the torch rule the
    fused Triton kernel reproduces bit for bit).
    """
    import torch
    from slimkv.llama3.prefill_ops import PrefillMetadata
    sys.path.insert(0, str(ROOT))
    from oracle.schedule import interleave_roles
    attn, (cos, sin) = _prefill_module(7)
    names = {'q': attn.q_proj, 'k': attn.k_proj, 'v': attn.v_proj, 'bq': attn.beacon_q_proj,
             'k_down': attn.beacon_k_down_proj, 'v_down': attn.beacon_v_down_proj,
             'k_up': attn.beacon_k_up_proj, 'v_up': attn.beacon_v_up_proj}
    for name, mod in names.items():
        out[f'prefill_w_{name}'] = mod.weight.detach().view(torch.int16).numpy()
        if mod.bias is not None:
            out[f'prefill_w_{name}_bias'] = mod.bias.detach().view(torch.int16).numpy()
    rng = np.random.default_rng(51)
    # (tag, previous chunk (raw count, remainder) or None, this chunk (raw count, remainder))
    cases = [('first', None, (13, 0)), ('second', (13, 0), (7, 1)), ('nobeacon', None, (2, 0)),
             ('long', None, (61, 3))]
    for tag, prev, cur in cases:
        roles, size, _ = interleave_roles(*cur, 4)
        window = np.concatenate([interleave_roles(*prev, 4)[0], roles]) if prev else roles
        n = len(roles)
        hidden = torch.from_numpy(rng.standard_normal((2, n, 128), dtype=np.float32)).to(torch.bfloat16)
        indices = torch.from_numpy(window)
        current = indices[-n:]
        attn._prefill_metadata = PrefillMetadata((current == 0).nonzero().flatten(),
                                                 (current != 0).nonzero().flatten(), indices, None, False)
        with torch.inference_mode():
            q, k, v, kl, vl = attn.qkv_proj_with_beacon(hidden, size, indices, return_latents=True)
            kv = k.view(2, n, 2, 32).transpose(1, 2)
            vv = v.view(2, n, 2, 32).transpose(1, 2)
            update = attn._incremental_cache(kv, vv, size, indices, (kl, vl))
        attn._prefill_metadata = None
        out[f'prefill_{tag}_roles'] = window
        out[f'prefill_{tag}_hidden'] = hidden.view(torch.int16).numpy()
        out[f'prefill_{tag}_query'] = q.view(torch.int16).numpy()
        out[f'prefill_{tag}_key'] = k.view(torch.int16).numpy()
        out[f'prefill_{tag}_value'] = v.view(torch.int16).numpy()
        out[f'prefill_{tag}_raw_indices'] = update.raw_indices.numpy()
        if size:
            out[f'prefill_{tag}_key_latents'] = update.key_latents.view(torch.int16).numpy()
            out[f'prefill_{tag}_value_latents'] = update.value_latents.view(torch.int16).numpy()
    # Prefill RoPE: the shapes of the reference's fused-rotary test.
    for tag, (batch, qlen, length, sink) in {'a': (1, 3, 3, 0), 'b': (2, 37, 129, 1), 'c': (4, 32, 65, 3)}.items():
        q = torch.from_numpy(rng.standard_normal((batch, 4, qlen, 32), dtype=np.float32) * 2).to(torch.bfloat16)
        k = torch.from_numpy(rng.standard_normal((batch, 2, length, 32), dtype=np.float32) * 2).to(torch.bfloat16)
        roles = (torch.arange(qlen) % 5 == 4).long()
        roles[::17] = 2
        positions = (torch.arange(length)[None] + 3 * torch.arange(batch)[:, None])
        attn.config.beacon_sink_size = sink
        with torch.inference_mode():
            qo, ko = attn._apply_rotary_with_beacon(q, k, positions, int((roles != 0).sum()), roles)
        out[f'prope_{tag}_q'] = q.view(torch.int16).numpy()
        out[f'prope_{tag}_k'] = k.view(torch.int16).numpy()
        out[f'prope_{tag}_roles'] = roles.numpy()
        out[f'prope_{tag}_pos'] = positions.numpy()
        out[f'prope_{tag}_sink'] = np.array(sink)
        out[f'prope_{tag}_qo'] = qo.contiguous().view(torch.int16).numpy()
        out[f'prope_{tag}_ko'] = ko.contiguous().view(torch.int16).numpy()
    out['prope_cos'] = cos.numpy()
    out['prope_sin'] = sin.numpy()


def gen_splits(out):
    from slimkv.llama3.paired_decode import original_splits
    rows = []
    for width in [128, 256, 320]:
        for keys in [1, 63, 64, 129, 1027, 8256, 16448, 32832, 131072]:
            for heads in [1, 8, 32, 64, 256]:
                for sms in [78, 132, 148]:
                    rows.append((width, keys, heads, sms, original_splits(width, keys, heads, sms)))
    out['splits'] = np.array(rows)


def gen_reconstruct(out):
    """``ReconstructionCache.materialize`` (slimkv/llama3/memory.py:26-48) with
    bf16 up-projections: the Beacon keys / values of the reconstruct backend."""
    import types
    import torch
    from slimkv.llama3.memory import ReconstructionCache
    for name, (seed, batch, n, rank, kv_heads, dim, bias) in {
            'qwen_r2': (31, 2, 70, 512, 2, 128, True), 'llama_r4': (32, 1, 45, 320, 2, 128, False)}.items():
        rng = np.random.default_rng(seed)
        lat_k = rng.standard_normal((batch, n, rank), dtype=np.float32) * 1.3
        lat_v = rng.standard_normal((batch, n, rank), dtype=np.float32) * 1.3
        mods = {}
        for kind, lat in (('k', lat_k), ('v', lat_v)):
            lin = torch.nn.Linear(rank, kv_heads * dim, bias=bias, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(torch.from_numpy(rng.standard_normal((kv_heads * dim, rank), dtype=np.float32) * 0.05))
                if bias:
                    lin.bias.copy_(torch.from_numpy(rng.standard_normal(kv_heads * dim, dtype=np.float32) * 0.1))
            mods[kind] = lin
        attn = types.SimpleNamespace(beacon_k_up_proj=mods['k'], beacon_v_up_proj=mods['v'],
                                     num_key_value_heads=kv_heads, head_dim=dim)
        for kind, lat in (('k', lat_k), ('v', lat_v)):
            hist = torch.from_numpy(lat).to(torch.bfloat16).unsqueeze(1)            # [B, 1, N, R]
            cache = ReconstructionCache(None, hist, None, None, None, kv_heads, dim, kind)
            with torch.no_grad():
                full = cache.materialize(attn)                                       # [B, Hkv, N, D] bf16
            out[f'{name}_lat_{kind}'] = hist.squeeze(1).view(torch.int16).numpy()
            out[f'{name}_w_{kind}'] = mods[kind].weight.detach().view(torch.int16).numpy()
            if bias:
                out[f'{name}_b_{kind}'] = mods[kind].bias.detach().view(torch.int16).numpy()
            out[f'{name}_full_{kind}'] = full.transpose(1, 2).contiguous().view(torch.int16).numpy()


def gen_prefill_attention(out):
    """The keys and values a prefill chunk attends over when its history is
    latent: ``ReconstructionCache.materialize(attention, current)``
    (slimkv/llama3/memory.py:26-48; the join of modeling_llama.py:1676-1681)
    with bf16 up-projections, then the chunk's causal attention over them in
    fp32 (torch SDPA with the bottom-right mask flash attention applies when
    the queries are the last tokens of the keys)."""
    import types
    import torch
    from slimkv.llama3.memory import ReconstructionCache
    for name, (seed, batch, sink, n, tokens, rank, heads, kv_heads, dim, bias) in {
            'llama_r4': (41, 2, 4, 200, 72, 320, 8, 2, 128, False),
            'qwen_r2': (42, 1, 4, 97, 40, 512, 10, 2, 128, True)}.items():
        rng = np.random.default_rng(seed)
        f32 = np.float32
        bf = lambda x: torch.from_numpy(np.ascontiguousarray(x, f32)).to(torch.bfloat16)
        q = bf(rng.standard_normal((batch, heads, tokens, dim), dtype=f32))
        sink_k = bf(rng.standard_normal((batch, kv_heads, sink, dim), dtype=f32))
        sink_v = bf(rng.standard_normal((batch, kv_heads, sink, dim), dtype=f32))
        cur_k = bf(rng.standard_normal((batch, kv_heads, tokens, dim), dtype=f32))
        cur_v = bf(rng.standard_normal((batch, kv_heads, tokens, dim), dtype=f32))
        lat = {kind: bf(rng.standard_normal((batch, 1, n, rank), dtype=f32) * 1.3) for kind in 'kv'}
        mods = {}
        for kind in 'kv':
            lin = torch.nn.Linear(rank, kv_heads * dim, bias=bias, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(torch.from_numpy(rng.standard_normal((kv_heads * dim, rank), dtype=f32) * 0.05))
                if bias:
                    lin.bias.copy_(torch.from_numpy(rng.standard_normal(kv_heads * dim, dtype=f32) * 0.1))
            mods[kind] = lin
        attn = types.SimpleNamespace(beacon_k_up_proj=mods['k'], beacon_v_up_proj=mods['v'],
                                     num_key_value_heads=kv_heads, head_dim=dim)
        full = {}
        for kind, sink_t, cur in (('k', sink_k, cur_k), ('v', sink_v, cur_v)):
            cache = ReconstructionCache(sink_t, lat[kind], None, None, None, kv_heads, dim, kind)
            with torch.no_grad():
                full[kind] = cache.materialize(attn, cur)                     # [B, Hkv, S + N + T, D] bf16
        keys = full['k'].shape[2]
        group = heads // kv_heads
        kf = full['k'].float().repeat_interleave(group, dim=1)
        vf = full['v'].float().repeat_interleave(group, dim=1)
        visible = torch.arange(keys)[None, :] <= (keys - tokens) + torch.arange(tokens)[:, None]
        scale = 1.0 / math.sqrt(dim)
        s = torch.einsum('bhtd,bhkd->bhtk', q.float(), kf) * scale
        s = s.masked_fill(~visible, float('-inf'))
        o = torch.softmax(s, -1) @ vf
        lse = torch.logsumexp(s, -1)
        i16 = lambda t: t.contiguous().view(torch.int16).numpy()
        out[f'{name}_q'] = i16(q.transpose(1, 2))                             # [B, T, H, D]
        out[f'{name}_sink_k'] = i16(sink_k.transpose(1, 2))                   # [B, S, Hkv, D]
        out[f'{name}_sink_v'] = i16(sink_v.transpose(1, 2))
        out[f'{name}_cur_k'] = i16(cur_k.transpose(1, 2))                     # [B, T, Hkv, D]
        out[f'{name}_cur_v'] = i16(cur_v.transpose(1, 2))
        for kind in 'kv':
            out[f'{name}_lat_{kind}'] = i16(lat[kind][:, 0])                  # [B, N, R]
            out[f'{name}_w_{kind}'] = i16(mods[kind].weight.detach())
            if bias:
                out[f'{name}_b_{kind}'] = i16(mods[kind].bias.detach())
        out[f'{name}_out'] = o.transpose(1, 2).numpy()                        # [B, T, H, D] fp32
        out[f'{name}_lse'] = lse.transpose(1, 2).numpy()                      # [B, T, H]


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument('--reference', required=True, help='path to a SlimKV source checkout')
    p.add_argument('--output', default=str(HERE / 'reference_golden.npz'))
    p.add_argument('--prefill-output', default=str(HERE / 'prefill_golden.npz'))
    p.add_argument('--reconstruct-output', default=str(HERE / 'reconstruct_golden.npz'))
    p.add_argument('--prefill-attention-output', default=str(HERE / 'prefill_attention_golden.npz'))
    p.add_argument('--only', choices=['decode', 'prefill', 'reconstruct', 'prefill_attention'], default=None,
                   help='write only the decode-side or only the prefill-side fixture file')
    args = p.parse_args()
    ref = Path(args.reference).resolve()
    sys.path[:0] = [str(_stubs()), str(ref), str(HERE), str(ROOT)]
    import torch
    torch.set_num_threads(4)
    from cases import config1_layer
    if args.only in (None, 'prefill_attention'):
        pa = {}
        gen_prefill_attention(pa)
        np.savez_compressed(args.prefill_attention_output, **pa)
        print('wrote', args.prefill_attention_output, sum(v.nbytes for v in pa.values()), 'bytes raw')
        if args.only == 'prefill_attention':
            return
    if args.only in (None, 'reconstruct'):
        rec = {}
        gen_reconstruct(rec)
        np.savez_compressed(args.reconstruct_output, **rec)
        print('wrote', args.reconstruct_output, sum(v.nbytes for v in rec.values()), 'bytes raw')
        if args.only == 'reconstruct':
            return
    if args.only != 'decode':
        pre = {}
        gen_prefill(pre)
        np.savez_compressed(args.prefill_output, **pre)
        print('wrote', args.prefill_output, sum(v.nbytes for v in pre.values()), 'bytes raw')
    if args.only == 'prefill':
        return
    out = {}
    gen_attention(out)
    gen_merge(out)
    gen_rope(out)
    gen_decode(out, 'c1', config1_layer())
    gen_decode(out, 'c1q2', config1_layer(length=2, history=1024, tail=7))
    gen_decode(out, 'small_bias', config1_layer(batch=2, length=2, history=40, tail=11, rank=16,
                                                hidden=256, heads=8, kv_heads=2, head_dim=32,
                                                bias=True, seed_w=5, seed_h=6))
    gen_decode(out, 'bias32', config1_layer(batch=2, length=2, history=300, tail=11, bias=True, seed_w=7,
                                            seed_h=8))
    gen_decode(out, 'qwen', config1_layer(batch=1, length=2, history=200, tail=5, rank=512, hidden=5120,
                                          heads=40, kv_heads=8, bias=True, seed_w=9, seed_h=10))
    gen_schedule(out, ref / 'tests')
    gen_model_decode(out, ref / 'tests')
    gen_interleave(out)
    gen_pages(out)
    gen_splits(out)
    np.savez_compressed(args.output, **out)
    print('wrote', args.output, sum(v.nbytes for v in out.values()), 'bytes raw')


if __name__ == '__main__':
    main()
