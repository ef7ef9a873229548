"""Rotate-half RoPE restated in numpy (test infrastructure only).

Follows micro-vllm's ``rotate_half`` and ``apply_rope``
(src/micro_vllm/model.py:101-123): ``x * cos + rotate_half(x) * sin`` with
``rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2])``, evaluated as torch
evaluates that tensor expression in the element type: each product is
rounded to the element type, then the sum is (fp32 operands widened exactly,
one IEEE float32 operation, one rounding to the storage type).

The tables are data: row p of cos/sin is the reference's ``rope_cos_sin`` at
position p (model.py:79-98), passed in as storage arrays.
"""
import numpy as np

from .dtypes import from_float32, to_float32


def rotate_half(x: np.ndarray) -> np.ndarray:
    """model.py:101-107 on float32 values: [a, b] -> [-b, a] over the last axis."""
    half = x.shape[-1] // 2
    return np.concatenate((-x[..., half:], x[..., :half]), axis=-1)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """RoPE of storage array x [..., D] with storage tables cos/sin broadcastable to x.

    Returns a storage array of ``dtype``.
    """
    xf = to_float32(x, dtype)
    cf = to_float32(cos, dtype)
    sf = to_float32(sin, dtype)
    with np.errstate(over='ignore', invalid='ignore'):
        first = to_float32(from_float32(np.multiply(xf, cf, dtype=np.float32), dtype), dtype)
        second = to_float32(from_float32(np.multiply(rotate_half(xf), sf, dtype=np.float32), dtype), dtype)
        return from_float32(np.add(first, second, dtype=np.float32), dtype)
