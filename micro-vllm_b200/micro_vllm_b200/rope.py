"""Rotary position embedding for the batched decode path.

``rope_tables`` builds the cos/sin tables of micro-vllm's ``rope_cos_sin``
(src/micro_vllm/model.py:79-98: fp32 inverse frequencies and angles,
duplicated halves, cos/sin, one cast to the activation dtype) for positions
0..num_positions-1, once per model; row p is the reference's table for
position p. ``apply_rope`` rotates rows on the GPU with libmvdecode.so's
``mv_apply_rope`` kernel, rounding each product and the sum to the element
type exactly as the reference's ``apply_rope`` expression does
(model.py:101-123). The decode step can also rotate q and the new K rows
inside the decode kernel (``paged_decode_with_append(..., rope=...)``).
"""
import math

import torch

from . import _native
from ._tensors import DTYPE_CODES, INDEX_CODES, current_stream_handle


def _check(condition, message):
    if not condition:
        raise RuntimeError(message)


def rope_tables(num_positions: int, head_dim: int, theta: float, *, dtype: torch.dtype,
                device: torch.device | str = 'cuda') -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin tables [num_positions, head_dim] of ``dtype`` on ``device``.

    Computed on the host in fp32 with the reference's operation order (so the
    values equal the reference's CPU tables bit for bit), then copied.
    """
    if head_dim <= 0 or head_dim % 2:
        raise ValueError('head_dim must be a positive even integer')
    if not math.isfinite(theta) or theta <= 0:
        raise ValueError('theta must be finite and positive')
    if type(num_positions) is not int or num_positions <= 0:
        raise ValueError('num_positions must be a positive integer')
    dimensions = torch.arange(0, head_dim, 2, dtype=torch.float32)
    inverse_freq = 1.0 / (theta ** (dimensions / head_dim))
    angles = torch.arange(num_positions).to(torch.float32).unsqueeze(-1) * inverse_freq
    duplicated = torch.cat((angles, angles), dim=-1)
    return (duplicated.cos().to(dtype).to(device).contiguous(),
            duplicated.sin().to(dtype).to(device).contiguous())


def check_tables(cos: torch.Tensor, sin: torch.Tensor, head_dim: int, dtype: torch.dtype,
                 device: torch.device) -> None:
    for table in (cos, sin):
        _check(isinstance(table, torch.Tensor) and table.is_cuda and table.dim() == 2
               and table.shape[1] == head_dim and table.shape[0] > 0 and table.is_contiguous(),
               'RoPE tables must be contiguous CUDA [positions, head_dim] tensors')
        _check(table.dtype == dtype and table.device == device,
               'RoPE tables must match the activation dtype and device')
    _check(cos.shape == sin.shape, 'RoPE cos and sin tables must have the same shape')


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
               positions: torch.Tensor | None = None, start: int = 0,
               positions_are_end: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rotate rows of x at their positions: x [B, H, T, D] or [B, H, D] (T = 1).

    Token t of sequence b sits at position start_b + t, where start_b is
    ``positions[b]`` (or ``positions[b] - T`` when ``positions_are_end``; for
    decode pass the context lengths including the new token) or ``start``.
    Positions without a table row give NaN rows. Returns out (a fresh tensor
    by default; out may be x for an in-place rotation).
    """
    three = x.dim() == 3
    x4 = x.unsqueeze(2) if three else x
    _check(isinstance(x, torch.Tensor) and x4.dim() == 4 and x4.numel() > 0,
           'x must be a nonempty [B, H, T, D] or [B, H, D] tensor')
    _check(x.is_cuda and x.dtype in DTYPE_CODES and not x.requires_grad,
           'x must be a CUDA float32, float16 or bfloat16 tensor without gradients')
    batch, heads, tokens, dim = x4.shape
    _check(dim % 2 == 0, 'head_dim must be even')
    _check(x4.stride(3) == 1 and all(x4.stride(d) >= 0 for d in range(3)),
           'x requires feature stride 1 and nonnegative outer strides')
    check_tables(cos, sin, dim, x.dtype, x.device)
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _check(out.shape == x.shape and out.dtype == x.dtype and out.device == x.device,
           'out must match x in shape, dtype and device')
    out4 = out.unsqueeze(2) if three else out
    _check(out4.stride(3) == 1, 'out requires feature stride 1')
    if positions is not None:
        _check(positions.is_cuda and positions.device == x.device and positions.dtype in INDEX_CODES
               and positions.shape == (batch,) and positions.is_contiguous(),
               'positions must be a contiguous [B] int32/int64 tensor on the device of x')
    lib = _native.library()
    with torch.cuda.device(x.device):
        _native.check(lib.mv_apply_rope(
            x4.data_ptr(), x4.stride(0), x4.stride(1), x4.stride(2),
            out4.data_ptr(), out4.stride(0), out4.stride(1), out4.stride(2),
            batch, heads, tokens, dim, cos.data_ptr(), sin.data_ptr(), cos.shape[0],
            positions.data_ptr() if positions is not None else None,
            INDEX_CODES[positions.dtype] if positions is not None else 0,
            _native.POSITIONS_END if positions_are_end else _native.POSITIONS_START, int(start),
            DTYPE_CODES[x.dtype], current_stream_handle(x.device)))
    return out
