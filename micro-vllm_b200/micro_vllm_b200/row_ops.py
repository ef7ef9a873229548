"""Fused row operations of the batched runtime's decode step (libmvdecode.so).

``rms_norm`` is the reference's RMSNorm (src/micro_vllm/model.py:25-41: fp32
statistics, normalised values cast back, then the scale) as one kernel per
call instead of a chain of elementwise launches; ``silu_mul`` is
``F.silu(gate) * up`` (model.py:150-165) on one fused gate/up projection
output, rounded step by step as the reference expression is.
"""
import torch

from . import _native
from ._tensors import DTYPE_CODES, current_stream_raw


def _check(condition, message):
    if not condition:
        raise RuntimeError(message)


def _rows(t):
    _check(t.is_cuda and t.dtype in DTYPE_CODES and t.dim() >= 1 and t.stride(-1) == 1,
           'row operations take CUDA float tensors with feature stride 1')
    _check(t.dim() == 2 or t.is_contiguous(), 'tensors other than [rows, width] must be contiguous')
    flat = t.view(-1, t.shape[-1]) if t.dim() != 2 else t
    _check(flat.dim() == 2 and (flat.shape[0] <= 1 or flat.stride(0) >= flat.shape[1]),
           'rows must not overlap')
    return flat


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """weight * to_dtype(x * rsqrt(mean(x^2, -1) + eps)) over the last dimension."""
    rows = _rows(x)
    _check(weight.shape == (x.shape[-1],) and weight.dtype == x.dtype and weight.is_contiguous()
           and weight.device == x.device, 'weight must be a contiguous [hidden] tensor of the input dtype')
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    o = _rows(out)
    _check(o.shape == rows.shape, 'out must match x')
    _native.check(_native.library().mv_rms_norm(
        rows.data_ptr(), rows.stride(0), weight.data_ptr(), o.data_ptr(), o.stride(0), rows.shape[0],
        rows.shape[1], float(eps), DTYPE_CODES[x.dtype], current_stream_raw(x.device.index)))
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(g) * u for the last dimension split as [g | u]."""
    rows = _rows(gate_up)
    _check(rows.shape[1] % 2 == 0, 'the last dimension must hold gate and up halves')
    width = rows.shape[1] // 2
    if out is None:
        out = torch.empty(gate_up.shape[:-1] + (width,), dtype=gate_up.dtype, device=gate_up.device)
    o = _rows(out)
    _check(o.shape == (rows.shape[0], width), 'out must be [..., width]')
    _native.check(_native.library().mv_silu_mul(
        rows.data_ptr(), rows.stride(0), o.data_ptr(), o.stride(0), rows.shape[0], width,
        DTYPE_CODES[gate_up.dtype], current_stream_raw(gate_up.device.index)))
    return out
