"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

from oracle.bf16 import bf16_bits


def to_bf16(x, device='cuda'):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device=device, dtype=torch.bfloat16)


def bits(t):
    """uint16 bit patterns of a bf16 tensor."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def assert_bits_equal(actual_bf16, expected_fp32):
    got = bits(actual_bf16)
    want = bf16_bits(expected_fp32)
    bad = np.nonzero(got.ravel() != want.ravel())[0]
    assert bad.size == 0, f'{bad.size} of {got.size} elements differ, first at {bad[:5]}'


# Parity bar.  fp32-accumulated outputs (the kernels' fp32 output mode): norm-wise
# relative error <= 2e-3 against the oracle.  bf16 outputs: rounding a value to
# bf16 alone costs a norm-wise relative error of 1.66e-3 (measured on Gaussian
# data), so their norm-wise bound is 3e-3, and every element must also meet the
# reference's own GPU validation tolerance (atol = rtol = 0.015,
# tools/validation/validate_fa2_decode.py:58).
REL_FP32 = 2e-3
REL_BF16 = 3e-3


def assert_attention_close(actual, expected, rel=None, atol=1.5e-2, rtol=1.5e-2):
    """Attention-output parity against the oracle; returns the norm-wise error."""
    if rel is None:
        rel = REL_FP32 if (torch.is_tensor(actual) and actual.dtype == torch.float32) else REL_BF16
    a = actual.float().cpu().numpy().astype(np.float64) if torch.is_tensor(actual) else np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    err = np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30)
    assert err <= rel, f'norm-wise relative error {err:.3e} > {rel}'
    np.testing.assert_allclose(a, e, atol=atol, rtol=rtol)
    return err


def assert_lse_close(actual, expected, atol=1e-3, masked=np.inf):
    a = actual.float().cpu().numpy() if torch.is_tensor(actual) else np.asarray(actual)
    e = np.asarray(expected, np.float64)
    masked_rows = np.isneginf(e)
    assert np.all(a[masked_rows] == masked), 'masked rows must carry the masked LSE value'
    np.testing.assert_allclose(a[~masked_rows], e[~masked_rows], atol=atol, rtol=1e-4)
