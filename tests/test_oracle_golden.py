"""Pin the CPU oracle against outputs of micro-vllm's own reference code.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py,
which runs the reference's PagedKVCache append/gather and causal_attention.
"""
import numpy as np
import pytest

from oracle import append_tokens, decode_float, decode_reference, to_float32
from oracle.dtypes import bf16_to_f32, f32_to_bf16
from tests.golden.cases import array_digest, input_digest, make_inputs
from tests.golden.make_golden import GOLDEN_CASES

GOLDEN_DIR = __import__('pathlib').Path(__file__).resolve().parent / 'golden'

# The oracle rounds once from fp64 where torch accumulates in its own order;
# allow that difference (fp32) or one unit in the last place (fp16/bf16).
PIN_TOLERANCE = {
    'float32': dict(rtol=2e-6, atol=1e-6),
    'float16': dict(rtol=2 ** -10, atol=2 ** -14),
    'bfloat16': dict(rtol=2 ** -7, atol=2 ** -12),
}


def load_fixture(name):
    with np.load(GOLDEN_DIR / f'{name}.npz') as data:
        return {key: data[key] for key in data.files}


def appended(inputs):
    key_pool = inputs['key_pool'].copy()
    value_pool = inputs['value_pool'].copy()
    starts = inputs['context_lens'].astype(np.int64) - 1
    append_tokens(key_pool, value_pool, inputs['key_new'], inputs['value_new'],
                  inputs['block_table'], starts)
    return key_pool, value_pool


@pytest.mark.parametrize('name', GOLDEN_CASES)
def test_inputs_regenerate_identically(name):
    fixture = load_fixture(name)
    assert input_digest(make_inputs(name)) == str(fixture['input_digest'])


@pytest.mark.parametrize('name', GOLDEN_CASES)
def test_append_oracle_is_bit_exact_against_reference(name):
    fixture = load_fixture(name)
    key_pool, value_pool = appended(make_inputs(name))
    assert array_digest(key_pool) == str(fixture['key_pool_digest'])
    assert array_digest(value_pool) == str(fixture['value_pool_digest'])


@pytest.mark.parametrize('name', GOLDEN_CASES)
def test_decode_oracle_matches_reference_outputs(name):
    fixture = load_fixture(name)
    inputs = make_inputs(name)
    dtype = str(fixture['dtype'])
    key_pool, value_pool = appended(inputs)
    ours = decode_reference(inputs['q'], key_pool, value_pool, inputs['block_table'],
                            inputs['context_lens'], dtype)
    np.testing.assert_allclose(to_float32(ours, dtype), to_float32(fixture['out'], dtype),
                               **PIN_TOLERANCE[dtype])


@pytest.mark.parametrize('name', GOLDEN_CASES)
def test_float_oracle_is_close_to_reference(name):
    """The unrounded parity oracle sits within the reference's own dtype error.

    The reference rounds scores to bf16 before the softmax (attention.py:87), so
    with the x8 K outliers its bf16 output drifts by up to ~0.1 from exact math.
    """
    fixture = load_fixture(name)
    inputs = make_inputs(name)
    dtype = str(fixture['dtype'])
    key_pool, value_pool = appended(inputs)
    dim = inputs['q'].shape[-1]
    exact = decode_float(inputs['q'], key_pool, value_pool, inputs['block_table'],
                         inputs['context_lens'], dim ** -0.5, dtype)
    reference = to_float32(fixture['out'], dtype)
    tolerance = {'float32': 1e-5, 'float16': 5e-3, 'bfloat16': 0.15}[dtype]
    assert np.max(np.abs(exact - reference)) <= tolerance


def test_bf16_conversion_round_trips_and_rounds_to_nearest_even():
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    widened = bf16_to_f32(bits)
    finite = ~np.isnan(widened)
    assert np.array_equal(f32_to_bf16(widened)[finite], bits[finite])
    # 1 + 2^-8 is the midpoint between 1 and 1 + 2^-7: ties go to the even value 1.0.
    assert f32_to_bf16(np.float32(1 + 2 ** -8)) == 0x3F80
    assert f32_to_bf16(np.float32(1 + 3 * 2 ** -8)) == 0x3F82
