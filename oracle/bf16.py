"""BF16 helpers for the CPU oracle (test infrastructure only).

bfloat16 is the upper half of an IEEE fp32 word.  Rounding from fp32 is
round-to-nearest-even on the dropped 16 bits, which is what PyTorch's
``tensor.to(torch.bfloat16)`` and CUDA's ``__float2bfloat16_rn`` do; NaN stays
NaN (quietened).
"""
import numpy as np


def bf16_bits(x):
    """fp32 array -> uint16 bf16 bit patterns, round to nearest even."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32)
    # uint32 arithmetic wraps only for bit patterns >= 0xFFFF8001, which are
    # NaNs and are replaced below.
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | np.uint32(0x40)).astype(np.uint16)
    return r


def from_bf16_bits(bits):
    """uint16 bf16 bit patterns -> fp32 values (exact)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def round_bf16(x):
    """Round fp32 values to the nearest bf16 value, returned as fp32."""
    return from_bf16_bits(bf16_bits(x))
