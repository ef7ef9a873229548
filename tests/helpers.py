"""Conversions between the oracle's numpy arrays and CUDA tensors, and tolerances."""
import numpy as np
import torch

from oracle import to_float32

TORCH_DTYPES = {'float32': torch.float32, 'float16': torch.float16, 'bfloat16': torch.bfloat16}


def to_torch(array, dtype_name=None, device='cuda'):
    array = np.ascontiguousarray(array)
    if dtype_name == 'bfloat16':
        return torch.from_numpy(array.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(array.copy()).to(device)


def to_numpy(tensor, dtype_name=None):
    tensor = tensor.detach().contiguous().cpu()
    if tensor.dtype == torch.bfloat16:
        return tensor.view(torch.int16).numpy().view(np.uint16).copy()
    return tensor.numpy().copy()


def as_float(tensor):
    """fp32 numpy copy of a CUDA tensor of any float dtype."""
    name = {torch.float32: 'float32', torch.float16: 'float16', torch.bfloat16: 'bfloat16'}[tensor.dtype]
    return to_float32(to_numpy(tensor), name)


def workload_tensors(inputs, device='cuda'):
    dtype = inputs['spec']['dtype']
    return dict(
        q=to_torch(inputs['q'], dtype, device),
        key_pool=to_torch(inputs['key_pool'], dtype, device),
        value_pool=to_torch(inputs['value_pool'], dtype, device),
        key_new=to_torch(inputs['key_new'], dtype, device),
        value_new=to_torch(inputs['value_new'], dtype, device),
        block_table=to_torch(inputs['block_table'], None, device),
        context_lens=to_torch(inputs['context_lens'], None, device),
    )


def assert_attention_close(actual, expected, dtype):
    """The parity bar: fp32 within 1e-5 relative (atol 1e-6 for values near 0);
    fp16 within the reference tests' 2e-3; bf16 within 2e-2 max-abs of the
    fp32/fp64 oracle. NaN must match NaN."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape
    assert np.array_equal(np.isnan(actual), np.isnan(expected)), 'NaN pattern differs'
    finite = ~np.isnan(expected)
    a, e = actual[finite], expected[finite]
    if dtype == 'float32':
        np.testing.assert_allclose(a, e, rtol=1e-5, atol=1e-6)
    elif dtype == 'float16':
        np.testing.assert_allclose(a, e, rtol=2e-3, atol=2e-3)
    else:
        err = np.max(np.abs(a - e)) if a.size else 0.0
        assert err <= 2e-2, f'bf16 max-abs error {err}'
