"""GPU parity of RoPE: the standalone kernel (mv_apply_rope) and RoPE fused into
the one-call decode step, against the reference's outputs and the oracle."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import append_tokens, apply_rope as oracle_rope, decode_float
from tests.golden.cases import make_inputs
from tests.golden.make_golden_rope import POSITIONS, ROPE_CASES
from tests.helpers import TORCH_DTYPES, as_float, assert_attention_close, to_numpy, to_torch, workload_tensors

pytestmark = pytest.mark.gpu

FIXTURE = Path(__file__).resolve().parent / 'golden' / 'rope_cases.npz'


def _bits_equal(a, b):
    a, b = a.contiguous(), b.contiguous()
    view = torch.int16 if a.element_size() == 2 else torch.int32
    return torch.equal(a.view(view), b.view(view))


def _tables(rows, dim, dtype):
    from micro_vllm_b200.rope import rope_tables
    return rope_tables(rows, dim, 1e6, dtype=TORCH_DTYPES[dtype], device='cuda')


@pytest.mark.parametrize('dtype,dim', ROPE_CASES)
def test_kernel_matches_the_reference_outputs(dtype, dim):
    from micro_vllm_b200.rope import apply_rope
    with np.load(FIXTURE) as f:
        data = {k: f[k] for k in f.files}
    cos, sin = _tables(int(POSITIONS.max()) + 1, dim, dtype)
    positions = torch.from_numpy(POSITIONS).cuda()
    tag = f'{dtype}_{dim}'
    for name in ('q', 'k'):
        x = to_torch(data[f'{tag}_{name}'], dtype)                # [positions, heads, D]
        out = apply_rope(x, cos, sin, positions=positions)        # one token per "sequence"
        expected = to_torch(data[f'{tag}_{name}_out'], dtype)
        assert _bits_equal(out, expected), name
        # In place gives the same bits.
        y = x.clone()
        apply_rope(y, cos, sin, positions=positions, out=y)
        assert _bits_equal(y, expected)


@pytest.mark.parametrize('dtype', ['float32', 'float16', 'bfloat16'])
def test_token_rows_positions_and_strides_against_the_oracle(dtype):
    from micro_vllm_b200.rope import apply_rope
    rng = np.random.default_rng(5)
    batch, heads, tokens, dim = 3, 5, 7, 64
    cos, sin = _tables(256, dim, dtype)
    base = torch.from_numpy(rng.standard_normal((batch, tokens, heads + 3, dim), dtype=np.float32))
    x = base.to(TORCH_DTYPES[dtype]).cuda().transpose(1, 2)[:, 1:heads + 1]   # strided [B, H, T, D]
    ends = torch.tensor([7, 100, 255], dtype=torch.int32, device='cuda')
    out = apply_rope(x, cos, sin, positions=ends, positions_are_end=True)
    cos_np, sin_np = to_numpy(cos), to_numpy(sin)
    x_np = to_numpy(x)
    for b, end in enumerate(ends.tolist()):
        pos = np.arange(end - tokens, end)
        expected = oracle_rope(x_np[b], cos_np[pos][None], sin_np[pos][None], dtype)
        assert np.array_equal(to_numpy(out[b]).view(np.uint8), expected.view(np.uint8))
    # Start positions and positions outside the table.
    out = apply_rope(x, cos, sin, start=250)
    values = as_float(out)
    assert np.isfinite(values[:, :, :6]).all() and np.isnan(values[:, :, 6:]).all()


@pytest.mark.parametrize('name', ['qwen7b_bf16_small', 'qwen72b_bf16_small', 'qwen05b_fp16',
                                  'qwen05b_fp32', 'edge_bs64_d64_bf16'])
@pytest.mark.parametrize('mode', [{}, dict(pages_per_split=4), dict(persistent=True), dict(force_simt=True)])
def test_fused_rope_step_equals_rotate_then_step_and_the_oracle(name, mode):
    from micro_vllm_b200 import cuda_attention
    from micro_vllm_b200.rope import apply_rope
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    dim = t['q'].shape[-1]
    cap = t['block_table'].shape[1] * t['key_pool'].shape[2]
    cos, sin = _tables(cap, dim, dtype)
    key, value = t['key_new'][:, :, 0], t['value_new'][:, :, 0]
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    out = cuda_attention.paged_decode_with_append(t['q'], key, value, *pools, t['block_table'],
                                                  t['context_lens'], rope=(cos, sin), **mode)
    # Reference order: rotate q and K at position len - 1, append, attend.
    q_rot = apply_rope(t['q'], cos, sin, positions=t['context_lens'], positions_are_end=True)
    k_rot = apply_rope(key, cos, sin, positions=t['context_lens'], positions_are_end=True)
    ref_pools = (t['key_pool'].clone(), t['value_pool'].clone())
    ref = cuda_attention.paged_decode_with_append(q_rot, k_rot, value, *ref_pools, t['block_table'],
                                                  t['context_lens'], **mode)
    torch.cuda.synchronize()
    assert _bits_equal(pools[0], ref_pools[0]) and _bits_equal(pools[1], ref_pools[1])
    assert _bits_equal(out, ref)
    # The oracle: numpy RoPE, append, decode.
    lens = inputs['context_lens'].astype(np.int64)
    cos_np, sin_np = to_numpy(cos), to_numpy(sin)
    q_np = oracle_rope(inputs['q'], cos_np[lens - 1][:, None], sin_np[lens - 1][:, None], dtype)
    k_np = oracle_rope(inputs['key_new'][:, :, 0], cos_np[lens - 1][:, None], sin_np[lens - 1][:, None], dtype)
    kp, vp = inputs['key_pool'].copy(), inputs['value_pool'].copy()
    append_tokens(kp, vp, k_np[:, :, None], inputs['value_new'], inputs['block_table'], lens - 1)
    assert np.array_equal(to_numpy(pools[0]).view(np.uint8), kp.view(np.uint8))
    expected = decode_float(q_np, kp, vp, inputs['block_table'], inputs['context_lens'], dim ** -0.5, dtype)
    assert_attention_close(as_float(out), expected, dtype)


def test_fused_rope_position_without_a_table_row_is_nan_and_touches_no_other_slot():
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    lens = inputs['context_lens']
    rows = int(lens.min())            # the shortest sequence's position len - 1 is the last row
    cos, sin = _tables(rows, 128, 'bfloat16')
    key, value = t['key_new'][:, :, 0], t['value_new'][:, :, 0]
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    out = as_float(cuda_attention.paged_decode_with_append(t['q'], key, value, *pools, t['block_table'],
                                                           t['context_lens'], rope=(cos, sin)))
    for b, length in enumerate(lens.tolist()):
        assert np.isnan(out[b]).all() == (length - 1 >= rows)
        assert np.isfinite(out[b]).all() == (length - 1 < rows)
    # Slots other than each sequence's new one are untouched.
    before = to_numpy(t['key_pool']).copy()
    after = to_numpy(pools[0])
    for b, length in enumerate(lens.tolist()):
        page = inputs['block_table'][b, (length - 1) // 16]
        before[page, :, (length - 1) % 16] = after[page, :, (length - 1) % 16]
    assert np.array_equal(before, after)


def test_bound_step_with_rope_matches_the_one_off_call():
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs('qwen72b_bf16_small')
    t = workload_tensors(inputs)
    cap = t['block_table'].shape[1] * 16
    cos, sin = _tables(cap, 128, 'bfloat16')
    key, value = t['key_new'][:, :, 0], t['value_new'][:, :, 0]
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    step = cuda_attention.PagedDecodeStep(*pools, t['block_table'], num_q_heads=t['q'].shape[1], rope=(cos, sin))
    out = step(t['q'], t['context_lens'], key=key, value=value)
    ref_pools = (t['key_pool'].clone(), t['value_pool'].clone())
    ref = cuda_attention.paged_decode_with_append(t['q'], key, value, *ref_pools, t['block_table'],
                                                  t['context_lens'], rope=(cos, sin))
    torch.cuda.synchronize()
    assert _bits_equal(out, ref) and _bits_equal(pools[0], ref_pools[0]) and _bits_equal(pools[1], ref_pools[1])
    with pytest.raises(RuntimeError, match='needs the new K/V rows'):
        step(t['q'], t['context_lens'])


@pytest.mark.parametrize('dtype', ['bfloat16', 'float16'])
def test_unaligned_rows_take_the_element_kernel_with_the_same_bits(dtype):
    """Rows whose stride is not a 16-byte multiple use the element-wise kernel;
    both kernels give the oracle's bits."""
    from micro_vllm_b200.rope import apply_rope
    cos, sin = _tables(64, 128, dtype)
    base = torch.randn(2, 3, 5, 129, device='cuda').to(TORCH_DTYPES[dtype])
    x = base[..., :128]                              # token stride 129 elements: not 16-byte aligned
    aligned = x.contiguous()
    a = apply_rope(x, cos, sin, start=7)
    b = apply_rope(aligned, cos, sin, start=7)
    assert _bits_equal(a, b)
    expected = oracle_rope(to_numpy(aligned), to_numpy(cos)[7:12][None, None], to_numpy(sin)[7:12][None, None], dtype)
    assert np.array_equal(to_numpy(a).view(np.uint8), expected.view(np.uint8))
