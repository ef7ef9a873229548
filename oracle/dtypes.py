"""Storage representations for the oracle (test infrastructure only).

numpy has no bfloat16, so bf16 tensors travel as uint16 bit patterns. float16
and float32 use numpy's own types. Conversions follow IEEE round-to-nearest-
even, which is what PyTorch's CPU casts do (c10/util/BFloat16.h
round_to_nearest_even; NaN becomes the canonical quiet NaN 0x7FC0).
"""
import numpy as np

# name -> numpy storage dtype
STORAGE_DTYPES = {
    'float32': np.float32,
    'float16': np.float16,
    'bfloat16': np.uint16,
}


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32 exactly."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 bit patterns with round-to-nearest-even."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    bits = values.view(np.uint32)
    with np.errstate(over='ignore'):
        bias = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
        rounded = ((bits + bias) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(values)
    if nan.any():
        rounded[nan] = np.uint16(0x7FC0)
    return rounded


def to_float32(array: np.ndarray, dtype: str) -> np.ndarray:
    """Exact float32 view of a tensor stored as ``dtype``."""
    if dtype == 'bfloat16':
        return bf16_to_f32(array)
    if dtype in ('float16', 'float32'):
        return np.asarray(array).astype(np.float32)
    raise ValueError(f'unsupported dtype {dtype!r}')


def from_float32(values: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the storage representation of ``dtype``."""
    values = np.asarray(values, dtype=np.float32)
    if dtype == 'bfloat16':
        return f32_to_bf16(values)
    if dtype == 'float16':
        return values.astype(np.float16)
    if dtype == 'float32':
        return values.copy()
    raise ValueError(f'unsupported dtype {dtype!r}')


def round_through(values: np.ndarray, dtype: str) -> np.ndarray:
    """Round to ``dtype`` and widen back to float32 (a cast there and back)."""
    return to_float32(from_float32(values, dtype), dtype)
