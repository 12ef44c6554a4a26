"""GPU parity of the split-KV decode attention (drop-in extension path).

Compares ``slimkv_attention_forward`` (through the C ABI, via the drop-in
``slimkv_fa2_decode_320`` module and the fp32-output mode) with the CPU
oracle's eager attention on the same seeded bf16 inputs.  Tolerances: fp32
outputs norm-wise relative error 2e-3; bf16 outputs 3e-3 norm-wise (bf16
rounding alone is 1.66e-3) and element-wise atol = rtol = 0.015; LSE atol 1e-3
(the reference's own GPU validation, tools/validation/validate_fa2_decode.py:58-59).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from cases import attention_case
from gpu_util import assert_attention_close, assert_lse_close, to_bf16

pytestmark = pytest.mark.gpu


def _run(c, splits=0, lengths=None):
    from slimkv_b200.extension import slimkv_fa2_decode_320 as ext
    q, k, v = to_bf16(c['q']), to_bf16(c['k']), to_bf16(c['v'])
    seqlens = None if lengths is None else torch.tensor(lengths, dtype=torch.int32, device='cuda')
    out, lse = ext.forward(q, k, v, c['scale'], c['causal'], splits, True, seqlens)
    torch.cuda.synchronize()
    ref, ref_lse = oracle.eager_attention(c['q'], c['k'], c['v'], c['scale'], c['causal'], lengths)
    return out, lse, ref, ref_lse


CASES = [
    # (seed, batch, queries, heads, kv_heads, keys, dk, dv, causal)
    (1, 1, 1, 32, 1, 1, 320, 320, False),
    (2, 1, 2, 32, 1, 1, 320, 320, True),        # first query sees no key
    (3, 1, 2, 32, 1, 129, 320, 320, True),
    (4, 2, 1, 8, 2, 257, 320, 320, False),
    (5, 2, 1, 32, 8, 1027, 128, 128, False),    # raw branch geometry
    (6, 3, 2, 32, 8, 63, 128, 128, True),
    (7, 2, 1, 32, 1, 2048, 320, 320, False),
    (8, 2, 2, 32, 1, 777, 192, 192, True),
    (9, 1, 1, 40, 8, 300, 128, 128, False),     # Qwen GQA group of 5
    (10, 2, 2, 40, 1, 200, 256, 256, True),     # 80 rows -> two row blocks
    (11, 4, 1, 32, 1, 65, 64, 64, False),
    (12, 2, 1, 16, 4, 130, 256, 256, False),
]


@pytest.mark.parametrize('spec', CASES, ids=lambda s: f'b{s[1]}q{s[2]}h{s[3]}kv{s[4]}n{s[5]}w{s[6]}')
@pytest.mark.parametrize('splits', [0, 1, 16])
def test_attention_matches_oracle(spec, splits):
    from slimkv_b200 import kernels
    c = attention_case(*spec)
    out, lse, ref, ref_lse = _run(c, splits)
    assert_attention_close(out, ref)
    assert_lse_close(lse, ref_lse)
    q, k, v = to_bf16(c['q']), to_bf16(c['k']), to_bf16(c['v'])
    out32 = torch.empty(q.shape[:3] + (v.shape[3],), dtype=torch.float32, device='cuda')
    kernels.attention_forward(q, k, v, c['scale'], c['causal'], splits, out=out32)
    assert_attention_close(out32, ref)


def test_cache_seqlens_truncate_each_row():
    c = attention_case(21, 3, 1, 32, 1, 600, 320, 320, False)
    out, lse, ref, ref_lse = _run(c, lengths=[600, 1, 333])
    assert_attention_close(out, ref)
    assert_lse_close(lse, ref_lse)


@pytest.mark.parametrize('stale', [float('nan'), float('inf')])
def test_cache_rows_past_cache_seqlens_are_ignored(stale):
    """Like the reference kernel, rows past a length never reach the output."""
    from slimkv_b200 import kernels
    c = attention_case(25, 3, 1, 32, 1, 600, 320, 320, False)
    lengths = [600, 1, 333]
    q, k, v = to_bf16(c['q']), to_bf16(c['k']), to_bf16(c['v'])
    for b, n in enumerate(lengths):
        k[b, n:] = stale
        v[b, n:] = stale
    seq = torch.tensor(lengths, dtype=torch.int32, device='cuda')
    for splits in (0, 1, 16):
        out, lse = kernels.attention_forward(q, k, v, c['scale'], False, splits, seq)
        assert torch.isfinite(out.float()).all()
        for b, n in enumerate(lengths):
            ref, ref_lse = oracle.eager_attention(c['q'][b:b + 1], c['k'][b:b + 1, :n], c['v'][b:b + 1, :n],
                                                  c['scale'], False)
            assert_attention_close(out[b:b + 1], ref)
            assert_lse_close(lse[b:b + 1], ref_lse)


def test_cache_seqlens_with_causal_pair():
    c = attention_case(22, 2, 2, 32, 1, 300, 320, 320, True)
    out, lse, ref, ref_lse = _run(c, lengths=[1, 257])
    assert_attention_close(out, ref)
    assert_lse_close(lse, ref_lse)


def test_shared_cache_with_zero_batch_stride():
    """Paired decode passes one cache expanded over two rows (stride 0)."""
    from slimkv_b200 import kernels
    c = attention_case(23, 1, 2, 32, 1, 257, 320, 320, False)
    q = to_bf16(c['q']).transpose(0, 1)                         # [2, 1, 32, 320]
    k, v = to_bf16(c['k']), to_bf16(c['v'])
    lengths = torch.tensor([256, 257], dtype=torch.int32, device='cuda')
    out, lse = kernels.attention_forward(q, k.expand(2, -1, -1, -1), v.expand(2, -1, -1, -1), c['scale'],
                                         False, 3, lengths)
    ref, ref_lse = oracle.eager_attention(c['q'], c['k'], c['v'], c['scale'], True)
    assert_attention_close(out.transpose(0, 1), ref)
    assert_lse_close(lse.squeeze(-1).transpose(0, 1).unsqueeze(0), ref_lse)


def test_masked_rows_use_fa2_positive_infinity():
    c = attention_case(24, 1, 2, 32, 1, 1, 320, 320, True)
    out, lse, _, _ = _run(c)
    assert torch.isinf(lse[..., 0]).all() and (lse[..., 0] > 0).all()
    assert (out[:, 0] == 0).all()


def test_strided_views_and_padding_like_reference_wrapper():
    """Real-rank views padded to the kernel width, as flash_forward does."""
    from slimkv_b200.extension import slimkv_fa2_decode_320 as ext
    c = attention_case(25, 2, 1, 32, 1, 300, 304, 312, False)
    pad = lambda x: torch.nn.functional.pad(to_bf16(x), (0, 320 - x.shape[-1]))
    storage = torch.zeros(2, 512, 1, 640, dtype=torch.bfloat16, device='cuda')
    storage[:, :300, :, :320] = pad(c['k'])
    storage[:, :300, :, 320:] = pad(c['v'])
    k, v = storage[:, :300, :, :320], storage[:, :300, :, 320:]
    out, lse = ext.forward(pad(c['q']), k, v, c['scale'])
    ref, ref_lse = oracle.eager_attention(c['q'], c['k'], c['v'], c['scale'])
    assert_attention_close(out[..., :312], ref)
    assert_lse_close(lse, ref_lse)


def test_library_error_is_raised_not_hidden():
    from slimkv_b200 import kernels, _lib
    q = torch.zeros(1, 3, 32, 128, dtype=torch.bfloat16, device='cuda')
    k = torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(_lib.SlimKVError):
        kernels.attention_forward(q, k, k, 0.1)
    assert _lib.device_status(clear=True) == 0
