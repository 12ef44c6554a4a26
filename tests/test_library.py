"""The C-ABI library loads on the CPU host and exports every declared symbol.

No compute calls here: only argument validation paths that reject input on
the host before any device work.
"""
import ctypes
import re
from pathlib import Path

import pytest

from slimkv_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / 'include' / 'slimkv_b200.h'


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r'\b(slimkv_[a-z0-9_]+)\s*\(', text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f'{name} has no ctypes signature'


def test_version_and_error_text():
    lib = _lib.load()
    assert lib.slimkv_version() >= 100
    assert isinstance(lib.slimkv_last_error(), bytes)


def _args(**kw):
    a = _lib.AttentionArgs()
    a.batch, a.queries, a.heads, a.kv_heads, a.keys = 1, 1, 32, 1, 64
    a.head_dim = a.value_dim = 320
    a.scale = 0.1
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize('bad,code', [
    (dict(queries=3), 1), (dict(heads=30, kv_heads=8), 1), (dict(keys=0), 1),
    (dict(head_dim=324), 2), (dict(value_dim=12), 2), (dict(batch=0), 1)])
def test_attention_rejects_invalid_arguments_before_launch(bad, code):
    lib = _lib.load()
    a = _args(**bad)
    assert lib.slimkv_attention_workspace_size(ctypes.byref(a)) == 0
    assert lib.slimkv_attention_forward(ctypes.byref(a), None, 0, None) == code
    assert lib.slimkv_last_error()


def test_attention_requires_workspace():
    lib = _lib.load()
    a = _args()
    assert lib.slimkv_attention_forward(ctypes.byref(a), None, 0, None) == 1   # null tensors first


def test_latent_decode_rejects_invalid_arguments():
    lib = _lib.load()
    a = _lib.LatentDecodeArgs()
    a.batch, a.length, a.heads, a.kv_heads, a.head_dim, a.rank_k, a.rank_v = 2, 1, 32, 8, 128, 320, 320
    a.raw_capacity, a.lat_capacity = 64, 64
    for field, value, code in [('length', 3, 1), ('head_dim', 64, 2), ('rank_k', 330, 2), ('heads', 31, 1),
                               ('raw_capacity', 0, 1)]:
        old = getattr(a, field)
        setattr(a, field, value)
        assert lib.slimkv_latent_decode_workspace_size(ctypes.byref(a)) == 0
        assert lib.slimkv_latent_decode(ctypes.byref(a), None, 0, None) == code, field
        setattr(a, field, old)


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, '_lib', None)
    monkeypatch.setattr(_lib, 'LIB_PATH', tmp_path / 'missing.so')
    with pytest.raises(ImportError):
        _lib.load()
