"""Drop-in replacement for the reference decode extension module.

Point ``SLIMKV_FA2_DECODE_EXTENSION_DIR`` at this directory and the
reference's ``importlib.import_module('slimkv_fa2_decode_320')``
(slimkv/llama3/fa2_decode.py:25-30, static_decode.py:20-29) loads this module
instead of the FA2 width-320 build.  ``forward`` keeps the signature, checks,
output layouts and the +inf LSE convention for fully masked rows of the
reference binding (kernels/fa2_decode/binding.cpp:35-130); the work runs in
the sm_100a kernels of ``libslimkv_b200.so``.
"""
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from slimkv_b200 import kernels as _kernels  # noqa: E402

supports_cache_seqlens = True


def forward(q, k, v, softmax_scale, causal=False, num_splits=0, pack_q=True, cache_seqlens=None):
    """BF16 decode attention: returns ``[out, lse]``.

    ``q [B, Q, H, W]``, ``k``/``v`` ``[B, N, Hkv, W]`` (arbitrary leading
    strides, contiguous last dimension; a stride-0 batch is allowed), Q in
    {1, 2}, causal only for Q == 2 (bottom-right).  ``out`` is BSHD bf16 and
    ``lse`` fp32 ``[B, H, Q]`` with +inf on rows that see no key.
    ``num_splits`` only changes the reduction partition; ``pack_q`` is
    accepted for signature compatibility (GQA packing is always used).
    """
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError('CUDA tensors required')
    if q.device != k.device or q.device != v.device:
        raise RuntimeError('Same device required')
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError('BSHD tensors required')
    width = q.shape[3]
    if k.shape[3] != width or v.shape[3] != width or width % 8 or width > 320:
        raise RuntimeError('Supported decode widths: multiples of 8 up to 320')
    if k.shape != v.shape or q.shape[0] != k.shape[0]:
        raise RuntimeError('Invalid K/V shape')
    if q.shape[1] not in (1, 2):
        raise RuntimeError('Decode supports one/two queries')
    if k.shape[1] <= 0:
        raise RuntimeError('Handle empty branches before calling FA2')
    if k.shape[2] <= 0 or q.shape[2] % k.shape[2]:
        raise RuntimeError('Invalid GQA head counts')
    causal = bool(causal) and q.shape[1] > 1
    out, lse = _kernels.attention_forward(q, k, v, softmax_scale, causal, num_splits, cache_seqlens,
                                          lse_masked_positive=True)
    return [out, lse]
