"""GPU checks of the fused row kernels against the reference's tensor expressions."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def reference_rms_norm(hidden, weight, eps):
    """src/micro_vllm/model.py:25-41."""
    hidden_fp32 = hidden.to(torch.float32)
    mean_square = hidden_fp32.pow(2).mean(dim=-1, keepdim=True)
    normalized = hidden_fp32 * torch.rsqrt(mean_square + eps)
    return weight * normalized.to(hidden.dtype)


ULP = {torch.float32: 2 ** -22, torch.float16: 2 ** -10, torch.bfloat16: 2 ** -7}


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize('shape', [(32, 1536), (3, 7, 256), (1, 33), (512, 4096), (2048, 1536), (4096, 896)])
def test_rms_norm_matches_the_reference_within_one_rounding(dtype, shape):
    from micro_vllm_b200.row_ops import rms_norm
    gen = torch.Generator(device='cuda').manual_seed(0)
    x = (torch.randn(shape, generator=gen, device='cuda') * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=gen, device='cuda')).to(dtype)
    out = rms_norm(x, w, 1e-6)
    expected = reference_rms_norm(x, w, 1e-6)
    diff = (out.float() - expected.float()).abs()
    # Summation order differs: within two roundings of the result; in 16-bit types the
    # final rounding absorbs the fp32 difference almost always.
    assert (diff <= ULP[dtype] * 2 * expected.float().abs() + 1e-30).all()
    if dtype != torch.float32:
        assert (diff == 0).float().mean() > 0.9


def test_rms_norm_strided_rows_and_out():
    from micro_vllm_b200.row_ops import rms_norm
    base = torch.randn(16, 300, device='cuda', dtype=torch.bfloat16)
    x = base[:, 22:278]
    w = torch.ones(256, device='cuda', dtype=torch.bfloat16)
    out = torch.full((16, 512), float('nan'), device='cuda', dtype=torch.bfloat16)
    rms_norm(x, w, 1e-5, out=out[:, :256])
    assert torch.isnan(out[:, 256:]).all()
    assert (out[:, :256].float() - reference_rms_norm(x, w, 1e-5).float()).abs().max() <= 2 ** -6


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_silu_mul_matches_the_reference_expression(dtype):
    from micro_vllm_b200.row_ops import silu_mul
    gen = torch.Generator(device='cuda').manual_seed(1)
    gate_up = (torch.randn(40, 2 * 8960 // 8, generator=gen, device='cuda') * 4).to(dtype)
    gate, up = gate_up.chunk(2, dim=-1)
    expected = F.silu(gate) * up
    out = silu_mul(gate_up)
    diff = (out.float() - expected.float()).abs()
    assert (diff <= ULP[dtype] * 2 * expected.float().abs() + 1e-30).all()
    assert (diff == 0).float().mean() > 0.99


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_odd_widths_and_unaligned_rows_take_the_element_kernels(dtype):
    """Widths that are not a multiple of a 16-byte chunk, rows at odd offsets."""
    from micro_vllm_b200.row_ops import rms_norm, silu_mul
    gen = torch.Generator(device='cuda').manual_seed(2)
    gate_up = (torch.randn(7, 2 * 37, generator=gen, device='cuda') * 3).to(dtype)
    gate, up = gate_up.chunk(2, dim=-1)
    diff = (silu_mul(gate_up).float() - (F.silu(gate) * up).float()).abs()
    assert (diff <= ULP[dtype] * 2 * (F.silu(gate) * up).float().abs() + 1e-30).all()
    x = (torch.randn(9, 101, generator=gen, device='cuda') * 2).to(dtype)
    w = torch.ones(101, device='cuda', dtype=dtype)
    expected = reference_rms_norm(x, w, 1e-6)
    assert ((rms_norm(x, w, 1e-6).float() - expected.float()).abs()
            <= ULP[dtype] * 2 * expected.float().abs() + 1e-30).all()
