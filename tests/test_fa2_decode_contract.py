"""Argument checks of the reference-contract ``decode`` (no GPU needed).

``slimkv_b200.fa2_decode.decode`` raises the reference's errors
(slimkv/llama3/fa2_decode.py:83-88) before touching a device, and refuses
what the fused kernel does not run (CPU tensors, another attention
``forward``) instead of falling back to a CPU path.
"""
import types

import pytest
import torch

from slimkv_b200 import fa2_decode


def _module(up=torch.nn.Linear):
    m = types.SimpleNamespace(
        beacon_k_up_proj=up(8, 16) if up is torch.nn.Linear else up(),
        beacon_v_up_proj=torch.nn.Linear(8, 16),
        config=types.SimpleNamespace(beacon_param=['q', 'k', 'v'], beacon_decode_backend='latent',
                                     _slimkv_decode_step=True),
        training=False)
    return m


def _cache():
    return types.SimpleNamespace(sink=None, history=None, raw=None, window=None, window_raw_indices=None)


@pytest.mark.parametrize('size,length', [(2, 3), (0, 2), (1, 1)])
def test_rejects_bad_beacon_sizes(size, length):
    with pytest.raises(ValueError, match='one raw token followed by at most one Beacon'):
        fa2_decode.decode(_module(), torch.zeros(1, length, 16), torch.zeros(1, 4, dtype=torch.long),
                          (_cache(), _cache(), size, None))


def test_rejects_non_linear_up_projections():
    with pytest.raises(ValueError, match='globally coupled Linear up projections'):
        fa2_decode.decode(_module(up=torch.nn.Identity), torch.zeros(1, 1, 16),
                          torch.zeros(1, 4, dtype=torch.long), (_cache(), _cache(), 0, None))


def test_rejects_cpu_tensors_instead_of_falling_back():
    with pytest.raises(ValueError, match='bf16 models on CUDA'):
        fa2_decode.decode(_module(), torch.zeros(1, 1, 16, dtype=torch.bfloat16),
                          torch.zeros(1, 4, dtype=torch.long), (_cache(), _cache(), 0, None))


def test_rejects_another_attention_forward():
    with pytest.raises(ValueError, match='forward=None'):
        fa2_decode.decode(_module(), torch.zeros(1, 1, 16), torch.zeros(1, 4, dtype=torch.long),
                          (_cache(), _cache(), 0, None), forward=lambda *a: None)


def test_eligibility_follows_the_reference():
    m = _module()
    hidden = torch.zeros(2, 2, 16)
    past = (_cache(), _cache(), 1, None)
    assert fa2_decode.eligible(m, hidden, past, False)
    assert not fa2_decode.eligible(m, hidden, past, True)                   # attention weights requested
    assert not fa2_decode.eligible(m, torch.zeros(2, 3, 16), past, False)   # more than raw + Beacon
    m.config.beacon_decode_backend = 'reconstruct'
    assert not fa2_decode.eligible(m, hidden, past, False)
    m.config.beacon_decode_backend = 'fa2'
    assert fa2_decode.eligible(m, hidden, past, False)
    assert not fa2_decode.eligible(m, hidden, (object(), object(), 1, None), False)   # not a latent cache
