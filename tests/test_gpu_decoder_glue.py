"""The decoder layer's element-wise steps of the batched runtime against the
reference modules' arithmetic in torch: ``LlamaRMSNorm.forward``
(slimkv/llama3/modeling_llama.py:79-95) and the gated product of
``LlamaMLP.forward`` (modeling_llama.py:97-113) on bf16 rows."""
import pytest
import torch
import torch.nn.functional as F

from slimkv_b200 import kernels

pytestmark = pytest.mark.gpu


def reference_rms_norm(x, weight, eps):
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return weight * h.to(x.dtype)


@pytest.mark.parametrize('rows,hidden,eps', [(32, 4096, 1e-5), (128, 5120, 1e-6), (3, 8192, 1e-5), (5, 136, 1e-6)])
def test_rms_norm_matches_the_reference_module(rows, hidden, eps):
    g = torch.Generator(device='cuda').manual_seed(rows + hidden)
    x = (torch.randn(rows, hidden, device='cuda', generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, device='cuda', generator=g)).to(torch.bfloat16)
    got = kernels.rms_norm(x, w, eps)
    want = reference_rms_norm(x, w, eps)
    # The mean of squares is summed in another order: at most one bf16 step apart.
    diff = (got.float() - want.float()).abs()
    assert (diff <= want.float().abs() * 2.0 ** -7 + 1e-30).all()
    assert (got == want).float().mean().item() > 0.99


def test_rms_norm_of_strided_rows_into_a_view():
    """The runtime normalises the raw-token rows x[:, 0] of [B, 2, H]."""
    x = torch.randn(16, 2, 4096, device='cuda').to(torch.bfloat16)
    w = torch.randn(4096, device='cuda').to(torch.bfloat16)
    out = torch.full((16, 4096), 7.0, device='cuda', dtype=torch.bfloat16)
    kernels.rms_norm(x[:, 0], w, 1e-5, out=out)
    diff = (out.float() - reference_rms_norm(x[:, 0], w, 1e-5).float()).abs()
    assert (diff <= reference_rms_norm(x[:, 0], w, 1e-5).float().abs() * 2.0 ** -7 + 1e-30).all()


@pytest.mark.parametrize('rows,inter', [(32, 14336), (128, 13824), (7, 24)])
def test_silu_mul_is_the_bf16_module_arithmetic(rows, inter):
    g = torch.Generator(device='cuda').manual_seed(rows * inter)
    gu = (torch.randn(rows, 2 * inter, device='cuda', generator=g) * 4).to(torch.bfloat16)
    got = kernels.silu_mul(gu)
    want = F.silu(gu[:, :inter]) * gu[:, inter:]
    assert torch.equal(got, want)


def test_glue_rejects_bad_shapes():
    from slimkv_b200._lib import SlimKVError
    x = torch.zeros(4, 12, device='cuda', dtype=torch.bfloat16)
    with pytest.raises(SlimKVError):
        kernels.rms_norm(x, torch.zeros(12, device='cuda', dtype=torch.bfloat16), 1e-5)
    with pytest.raises(SlimKVError):
        kernels.silu_mul(torch.zeros(4, 12, device='cuda', dtype=torch.bfloat16))
