"""Pin the prefill-attention restatement (``oracle/prefill_attention.py``) to
the reference: ``tests/golden/make_golden.py`` (``gen_prefill_attention``)
joined sinks, materialised history and the chunk's keys with the reference's
own ``ReconstructionCache.materialize`` (slimkv/llama3/memory.py:26-48, bf16
up-projections) and attended with the bottom-right causal mask in fp32."""
from pathlib import Path

import numpy as np
import pytest

from oracle.bf16 import from_bf16_bits
from oracle.prefill_attention import prefill_attention

GOLDEN = np.load(Path(__file__).parent / 'golden' / 'prefill_attention_golden.npz')


def case(name):
    g = {k[len(name) + 1:]: v for k, v in GOLDEN.items() if k.startswith(name + '_')}
    f = {k: (from_bf16_bits(v.view(np.uint16)) if v.dtype == np.int16 else v) for k, v in g.items()}
    return f


@pytest.mark.parametrize('name', ['llama_r4', 'qwen_r2'])
def test_oracle_matches_the_reference_join(name):
    c = case(name)
    B, T, H, D = c['q'].shape
    for b in range(B):
        out, lse = prefill_attention(c['q'][b], c['sink_k'][b], c['sink_v'][b], c['lat_k'][b], c['lat_v'][b],
                                     c['w_k'], c['w_v'], c['cur_k'][b], c['cur_v'][b], 1.0 / np.sqrt(D),
                                     c.get('b_k'), c.get('b_v'), bf16_history=True)
        # The reference rounds each materialised key / value to bf16 after an
        # fp32 dot product: a rare 1-ulp difference in one of them moves the
        # rows that weight it by ~1e-4; the whole output agrees to 2e-5.
        rel = np.linalg.norm(out - c['out'][b]) / np.linalg.norm(c['out'][b])
        assert rel <= 2e-5, rel
        np.testing.assert_allclose(out, c['out'][b], rtol=1e-3, atol=1e-3)
        np.testing.assert_allclose(lse, c['lse'][b], rtol=1e-5, atol=1e-4)


def test_bf16_history_rounding_is_visible():
    """Without the bf16 rounding of the materialised keys the restatement
    misses the reference by more than fp32 noise: the golden pins it."""
    c = case('llama_r4')
    D = c['q'].shape[-1]
    out, _ = prefill_attention(c['q'][0], c['sink_k'][0], c['sink_v'][0], c['lat_k'][0], c['lat_v'][0], c['w_k'],
                               c['w_v'], c['cur_k'][0], c['cur_v'][0], 1.0 / np.sqrt(D))
    assert np.abs(out - c['out'][0]).max() > 1e-4
