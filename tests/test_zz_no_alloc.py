"""The allocation-free attention entry point agrees with the workspace one.

``slimkv_attention_forward_noalloc`` serves callers that cannot allocate
device memory (for instance a host that reaches the library through an FFI
with no CUDA allocator of its own, or an engine that reserved all device
memory up front): its split scratch is a fixed 16 MiB array inside the
library.  Two calls in a row, with different shapes, must match the regular
``slimkv_attention_forward`` (which uses a caller workspace) within the
attention parity tolerance.  This file is collected last on purpose, and it
also passes when run alone in a fresh process.
"""
import pytest
import torch

from cases import attention_case
from gpu_util import assert_attention_close, assert_lse_close, to_bf16

pytestmark = pytest.mark.gpu


def _pair(spec, lengths=None):
    from slimkv_b200 import kernels
    c = attention_case(*spec)
    q, k, v = to_bf16(c['q']), to_bf16(c['k']), to_bf16(c['v'])
    seqlens = None if lengths is None else torch.tensor(lengths, dtype=torch.int32, device='cuda')
    ref, ref_lse = kernels.attention_forward(q, k, v, c['scale'], c['causal'], 0, seqlens)
    out = torch.full_like(ref, float('nan'))
    lse = torch.full_like(ref_lse, float('nan'))
    kernels.attention_forward_noalloc(q, k, v, c['scale'], out, lse, c['causal'], 0, seqlens)
    torch.cuda.synchronize()
    return out, lse, ref, ref_lse


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    from slimkv_b200 import _lib
    # Call 1: latent-width decode over one shared KV head.
    out, lse, ref, ref_lse = _pair((31, 4, 1, 32, 1, 1500, 320, 320, False), lengths=[1500, 7, 900, 1])
    assert_attention_close(out, ref.float().cpu().numpy())
    assert_lse_close(lse, ref_lse.cpu().numpy().astype('float64'), masked=float('inf'))
    # Call 2 reuses the same static scratch with a different shape (GQA, causal pair).
    out, lse, ref, ref_lse = _pair((32, 3, 2, 32, 8, 700, 128, 128, True))
    assert_attention_close(out, ref.float().cpu().numpy())
    assert_lse_close(lse, ref_lse.cpu().numpy().astype('float64'), masked=float('inf'))
    assert _lib.device_status(clear=True) == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    from slimkv_b200 import kernels, _lib
    q = torch.zeros(64, 2, 32, 320, dtype=torch.bfloat16, device='cuda')
    k = torch.zeros(64, 1024, 8, 320, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(64, 2, 32, 320, dtype=torch.bfloat16, device='cuda')
    lse = torch.empty(64, 32, 2, dtype=torch.float32, device='cuda')
    with pytest.raises(_lib.SlimKVError, match='static|scratch'):
        kernels.attention_forward_noalloc(q, k, k, 0.1, out, lse, num_splits=8)
