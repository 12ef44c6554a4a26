"""Stand-ins for the reference's attention module and cache in GPU tests.

``slimkv_b200.fa2_decode.decode`` reads a reference ``LlamaAttention``
(slimkv/llama3/modeling_llama.py:181-277) and its ``ReconstructionCache``
(slimkv/llama3/memory.py:10-48) by attribute.  The reference cannot be
imported on the GPU box, so these classes carry the same attribute names and
semantics: ``nn.Linear`` projections (biases as ``attention_bias`` gives
them), a table-based rotary embedding named like the reference's
``Llama3RotaryEmbedding``, ``o_proj_with_beacon`` without a Beacon o_proj
(``beacon_param`` of q, k, v; modeling_llama.py:1369-1382), and a cache with
``sink / history / raw / window / window_raw_indices`` views.
"""
import types

import numpy as np
import torch

from slimkv_b200.rope import LLAMA3_SCALING, rope_tables


class Llama3RotaryEmbedding:
    """Rotary tables with the reference's attribute names (fp32, CPU-built)."""

    def __init__(self, head_dim, theta, positions, scaling, device):
        self.cos_cached, self.sin_cached = rope_tables(head_dim, theta, positions, scaling, device)
        self.max_seq_len_cached = positions


class Attention(torch.nn.Module):
    """A reference-shaped latent attention module built from
    ``cases.config1_layer`` weights (rounded to bf16), on the device."""

    def __init__(self, case, device, theta=500000.0, scaling=LLAMA3_SCALING, positions=8192):
        super().__init__()
        w, bias = case['weights'], case['bias']
        H, heads, kv, d, R = case['hidden_size'], case['heads'], case['kv_heads'], case['head_dim'], case['rank']

        def lin(name, out, inp, bname=None):
            m = torch.nn.Linear(inp, out, bias=bname is not None and bias, device=device, dtype=torch.bfloat16)
            with torch.no_grad():
                m.weight.copy_(torch.from_numpy(w[name]))
                if m.bias is not None:
                    m.bias.copy_(torch.from_numpy(w[bname]))
            return m

        self.q_proj = lin('q_proj', heads * d, H, 'q_bias')
        self.k_proj = lin('k_proj', kv * d, H, 'k_bias')
        self.v_proj = lin('v_proj', kv * d, H, 'v_bias')
        self.o_proj = lin('o_proj', H, heads * d, 'o_bias')
        self.beacon_q_proj = lin('beacon_q_proj', heads * d, H, 'beacon_q_bias')
        self.beacon_k_down_proj = lin('k_down', R, H)
        self.beacon_v_down_proj = lin('v_down', R, H)
        self.beacon_k_up_proj = lin('k_up', kv * d, R, 'k_up_bias')
        self.beacon_v_up_proj = lin('v_up', kv * d, R, 'v_up_bias')
        self.rotary_emb = Llama3RotaryEmbedding(d, theta, positions, scaling, device)
        self.config = types.SimpleNamespace(beacon_param=['q', 'k', 'v'], beacon_decode_backend='latent',
                                            _slimkv_decode_step=True)
        self.num_heads, self.num_key_value_heads, self.head_dim, self.hidden_size = heads, kv, d, H
        self.num_key_value_groups = heads // kv
        self.eval()

    def _use_shared_kv_down_proj(self):
        return False

    def o_proj_with_beacon(self, attn_output, beacon_size, beacon_indices):
        return self.o_proj(attn_output)


def cache_pair(case, device, ratio=4):
    """Reference-layout caches of a ``config1_layer`` case: pre-RoPE sink and
    raw tail ``[B, Hkv, n, D]``, latents ``[B, 1, n, R]`` (bf16), the raw
    tail's window indices and the step's role list."""
    bf = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(device=device, dtype=torch.bfloat16)
    T, L = case['tail'], case['length']
    size = L - 1

    def bhsd(x):
        return None if x.shape[1] == 0 else bf(x).transpose(1, 2).contiguous()

    def lat(x):
        return None if x.shape[1] == 0 else bf(x)[:, None].contiguous()

    raw_idx = (torch.arange(T) + torch.arange(T) // ratio).to(device) if T else None
    n_win = case['win_k'].shape[1]
    roles = torch.zeros(T + n_win + 1 + size, dtype=torch.long, device=device)
    if T:
        roles[ratio::ratio + 1] = 1
    if size:
        roles[-1] = 1
    pk = types.SimpleNamespace(sink=bhsd(case['sink_k']), history=lat(case['hist_k']), raw=bhsd(case['tail_k']),
                               window=lat(case['win_k']), window_raw_indices=raw_idx)
    pv = types.SimpleNamespace(sink=bhsd(case['sink_v']), history=lat(case['hist_v']), raw=bhsd(case['tail_v']),
                               window=lat(case['win_v']), window_raw_indices=raw_idx)
    return pk, pv, size, roles
