"""ctypes binding of libmvdecode.so (declared in include/mvdecode.h).

The library is loaded on first use, never at import, and there is no fallback:
if it is missing or fails to load, every entry point raises.
"""
import ctypes
from functools import lru_cache
from pathlib import Path

import os

# MVDECODE_LIBRARY may name another build of the same library (e.g. a tuning variant).
LIB_PATH = Path(os.environ.get('MVDECODE_LIBRARY',
                               Path(__file__).resolve().parent / 'lib' / 'libmvdecode.so'))

MV_ABI_VERSION = 1
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
INDEX_I32, INDEX_I64 = 0, 1
POSITIONS_START, POSITIONS_END = 0, 1
FLAG_FORCE_SIMT = 1
FLAG_PERSISTENT = 2
FLAG_FUSED_MERGE = 4
FLAG_CLUSTER = 8
FLAG_WIDE = 16
FLAG_CHUNK_ROWS = 32
FLAG_CHUNK_MMA_SYNC = 64
FLAG_CUDA_CORE_MATH = 128
FLAG_STREAM = 256
FLAG_SPLIT_GRID = 512
PATH_SIMT, PATH_TMA_MMA, PATH_TMA_MMA_PERSISTENT, PATH_TMA_MMA_CLUSTER, PATH_TMA_MMA_STREAM = 0, 1, 2, 3, 4
PATH_NAMES = {0: 'simt', 1: 'tma_mma', 2: 'tma_mma_persistent', 3: 'tma_mma_cluster', 4: 'tma_mma_stream'}
DEVICE_STATUS_WAIT_TIMEOUT = 1
DEVICE_STATUS_BAD_PAGE_ID = 2

MV_OK = 0
STATUS_NAMES = {
    1: 'invalid argument',
    2: 'unsupported',
    3: 'workspace too small',
    4: 'CUDA error',
}

EXPORTED_SYMBOLS = (
    'mv_abi_version', 'mv_last_error', 'mv_paged_decode_workspace_size',
    'mv_paged_decode_plan', 'mv_paged_decode', 'mv_write_paged_kv',
    'mv_device_status', 'mv_clear_device_status', 'mv_paged_decode_append', 'mv_apply_rope',
    'mv_rms_norm', 'mv_silu_mul', 'mv_contiguous_decode_plan', 'mv_contiguous_decode',
    'mv_paged_chunk_workspace_size', 'mv_paged_chunk_attention', 'mv_selftest_wait_timeout',
    'mv_paged_decode_step_args',
)

_i32, _i64, _u32, _vp, _sz, _f32 = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32,
                                    ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float)

class MvDecodeStepArgs(ctypes.Structure):
    """MvDecodeStepArgs of include/mvdecode.h: every field 8 bytes, no padding."""
    _fields_ = [(name, kind) for names, kind in (
        (('q',), _vp), (('q_stride_seq', 'q_stride_head'), _i64),
        (('key',), _vp), (('key_stride_seq', 'key_stride_head'), _i64),
        (('value',), _vp), (('value_stride_seq', 'value_stride_head'), _i64),
        (('rope_cos', 'rope_sin'), _vp), (('rope_rows',), _i64),
        (('k_cache', 'v_cache'), _vp), (('num_blocks', 'num_kv_heads', 'block_size', 'head_dim'), _i64),
        (('block_table',), _vp), (('block_table_type', 'block_table_stride', 'blocks_per_seq'), _i64),
        (('context_lens',), _vp), (('context_lens_type', 'max_context_len', 'batch', 'num_q_heads'), _i64),
        (('scale',), ctypes.c_double),
        (('out',), _vp), (('out_stride_seq', 'out_stride_head'), _i64),
        (('workspace',), _vp), (('workspace_bytes',), ctypes.c_uint64), (('pages_per_split',), _i64),
        (('flags',), ctypes.c_uint64), (('dtype',), _i64)) for name in names]


_SIGNATURES = {
    'mv_paged_decode_step_args': (ctypes.c_int, [ctypes.POINTER(MvDecodeStepArgs), _vp]),
    'mv_abi_version': (ctypes.c_int, []),
    'mv_last_error': (ctypes.c_char_p, []),
    'mv_paged_decode_workspace_size': (
        ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _i64, _i32, _u32, _i32,
                       ctypes.POINTER(_sz)]),
    'mv_paged_decode_plan': (
        ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _i64, _i32, _u32, _i32, _vp, _vp,
                       ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    'mv_paged_decode': (
        ctypes.c_int, [_vp, _i64, _i64,            # q, strides
                       _vp, _vp, _i64,             # k_cache, v_cache, num_blocks
                       _i32, _i32, _i32,           # kv heads, block size, head dim
                       _vp, _i32, _i64, _i64,      # block table, type, stride, blocks/seq
                       _vp, _i32, _i64,            # context lens, type, max context len
                       _i32, _i32, _f32,           # batch, q heads, scale
                       _vp, _i64, _i64,            # out, strides
                       _vp, _sz, _i32, _u32, _i32, _vp]),  # workspace, bytes, pps, flags, dtype, stream
    'mv_write_paged_kv': (
        ctypes.c_int, [_vp, _i64, _i64, _i64,      # key, strides
                       _vp, _i64, _i64, _i64,      # value, strides
                       _vp, _vp, _i64,             # caches, num_blocks
                       _i32, _i32, _i32,           # kv heads, block size, head dim
                       _vp, _i32, _i64, _i64,      # block table, type, stride, blocks/seq
                       _vp, _i32, _i32, _i64,      # positions, type, kind, start
                       _i32, _i32, _i32, _vp]),    # batch, tokens, dtype, stream
    'mv_paged_decode_append': (
        ctypes.c_int, [_vp, _i64, _i64,            # q, strides
                       _vp, _i64, _i64,            # new key rows, strides
                       _vp, _i64, _i64,            # new value rows, strides
                       _vp, _vp, _i64,             # RoPE cos, sin tables, rows
                       _vp, _vp, _i64,             # k_cache, v_cache, num_blocks
                       _i32, _i32, _i32,           # kv heads, block size, head dim
                       _vp, _i32, _i64, _i64,      # block table, type, stride, blocks/seq
                       _vp, _i32, _i64,            # context lens, type, max context len
                       _i32, _i32, _f32,           # batch, q heads, scale
                       _vp, _i64, _i64,            # out, strides
                       _vp, _sz, _i32, _u32, _i32, _vp]),  # workspace, bytes, pps, flags, dtype, stream
    'mv_apply_rope': (
        ctypes.c_int, [_vp, _i64, _i64, _i64,      # x, strides
                       _vp, _i64, _i64, _i64,      # out, strides
                       _i32, _i32, _i32, _i32,     # batch, heads, tokens, head dim
                       _vp, _vp, _i64,             # cos, sin tables, rows
                       _vp, _i32, _i32, _i64,      # positions, type, kind, start
                       _i32, _vp]),                # dtype, stream
    'mv_rms_norm': (ctypes.c_int, [_vp, _i64, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp]),
    'mv_paged_chunk_workspace_size': (
        ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _u32, _i32, ctypes.POINTER(_sz)]),
    'mv_paged_chunk_attention': (
        ctypes.c_int, [_vp, _i64, _i64, _i64,      # q, strides (sequence, token, head)
                       _vp, _vp, _i64,             # k_cache, v_cache, num_blocks
                       _i32, _i32, _i32,           # kv heads, block size, head dim
                       _vp, _i32, _i64, _i64,      # block table, type, stride, blocks/seq
                       _vp, _i32, _i64,            # context lens, type, max context len
                       _i32, _i32, _i32, _f32,     # batch, tokens, q heads, scale
                       _vp, _i64, _i64, _i64,      # out, strides (sequence, token, head)
                       _vp, _sz, _i32, _u32, _i32, _vp]),  # workspace, bytes, pps, flags, dtype, stream
    'mv_contiguous_decode_plan': (
        ctypes.c_int, [_vp, _i64, _i64, _i64,      # k_cache, strides (sequence, head, token)
                       _vp, _i64, _i64, _i64,      # v_cache, strides
                       _i64, _i32, _i32, _i64,     # cache_len, kv heads, head dim, max context len
                       _i32, _i32, _i32, _u32, _i32,  # batch, q heads, pps, flags, dtype
                       ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                       ctypes.POINTER(_sz)]),
    'mv_contiguous_decode': (
        ctypes.c_int, [_vp, _i64, _i64,            # q, strides
                       _vp, _i64, _i64, _i64,      # k_cache, strides
                       _vp, _i64, _i64, _i64,      # v_cache, strides
                       _i64, _i32, _i32,           # cache_len, kv heads, head dim
                       _vp, _i32, _i64,            # context lens, type, max context len
                       _i32, _i32, _f32,           # batch, q heads, scale
                       _vp, _i64, _i64,            # out, strides
                       _vp, _sz, _i32, _u32, _i32, _vp]),  # workspace, bytes, pps, flags, dtype, stream
    'mv_silu_mul': (ctypes.c_int, [_vp, _i64, _vp, _i64, _i64, _i32, _i32, _vp]),
    'mv_device_status': (ctypes.c_int, [_i32, ctypes.POINTER(_u32)]),
    'mv_clear_device_status': (ctypes.c_int, [_i32]),
    'mv_selftest_wait_timeout': (ctypes.c_int, [ctypes.c_uint64, _vp]),
}


class NativeError(RuntimeError):
    """A libmvdecode entry point returned a non-OK status."""

    def __init__(self, status, message):
        super().__init__(f'{message} ({STATUS_NAMES.get(status, "status %d" % status)})')
        self.status = status


@lru_cache(maxsize=1)
def library() -> ctypes.CDLL:
    """Load libmvdecode.so once; raise if it is absent or incompatible."""
    if not LIB_PATH.exists():
        raise RuntimeError(
            f'{LIB_PATH} is not built: run `python -m micro_vllm_b200.build` '
            '(or __graft_entry__.build()) before using the CUDA kernels')
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    version = lib.mv_abi_version()
    if version != MV_ABI_VERSION:
        raise RuntimeError(f'libmvdecode ABI {version}, expected {MV_ABI_VERSION}')
    return lib


def check(status: int) -> None:
    if status != MV_OK:
        message = library().mv_last_error().decode(errors='replace')
        raise NativeError(status, message)


def call(name: str, *args) -> None:
    check(getattr(library(), name)(*args))
