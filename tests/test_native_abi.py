"""CPU checks of the C ABI: the library builds, loads, and exports what the header declares."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'mvdecode.h'


def _library():
    from micro_vllm_b200 import _native, build
    if build.is_stale():
        build.build()
    return _native.library()


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r'^MV_API\s+[\w\s\*]+?\b(mv_\w+)\s*\(', text, flags=re.MULTILINE)


def declared_constants():
    text = HEADER.read_text()
    return {name: int(value.rstrip('u'), 0) for name, value in
            re.findall(r'^#define\s+(MV_[A-Z0-9_]+)\s+(\d+u?)\b', text, flags=re.MULTILINE)}


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    assert set(names) == {
        'mv_abi_version', 'mv_last_error', 'mv_paged_decode_workspace_size',
        'mv_paged_decode_plan', 'mv_paged_decode', 'mv_write_paged_kv',
        'mv_device_status', 'mv_clear_device_status', 'mv_paged_decode_noalloc',
        'mv_paged_decode_append', 'mv_apply_rope', 'mv_rms_norm', 'mv_silu_mul',
        'mv_contiguous_decode_plan', 'mv_contiguous_decode', 'mv_paged_chunk_workspace_size',
        'mv_paged_chunk_attention', 'mv_selftest_wait_timeout', 'mv_paged_decode_step_args'}


def test_step_args_struct_matches_the_header():
    """MvDecodeStepArgs: the ctypes mirror has the header's fields, in order, 8 bytes each."""
    import ctypes
    from micro_vllm_b200 import _native
    body = re.search(r'typedef struct MvDecodeStepArgs \{(.*?)\} MvDecodeStepArgs;', HEADER.read_text(), re.S).group(1)
    names = []
    for decl in body.replace('\n', ' ').split(';'):
        decl = decl.strip()
        if decl:
            names.append(re.findall(r'(\w+)\s*$', decl)[0])
    assert names == [name for name, _ in _native.MvDecodeStepArgs._fields_]
    assert ctypes.sizeof(_native.MvDecodeStepArgs) == 8 * len(names)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.mv_abi_version() == declared_constants()['MV_ABI_VERSION']


def test_only_declared_symbols_are_exported():
    import subprocess
    from micro_vllm_b200 import _native
    _library()
    out = subprocess.run(['nm', '-D', '--defined-only', str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if ' T ' in line}
    assert {name for name in exported if name.startswith('mv_')} == set(declared_functions())


def test_python_binding_constants_match_the_header():
    from micro_vllm_b200 import _native
    constants = declared_constants()
    assert constants['MV_DTYPE_F32'] == _native.DTYPE_F32
    assert constants['MV_DTYPE_F16'] == _native.DTYPE_F16
    assert constants['MV_DTYPE_BF16'] == _native.DTYPE_BF16
    assert constants['MV_INDEX_I32'] == _native.INDEX_I32
    assert constants['MV_INDEX_I64'] == _native.INDEX_I64
    assert constants['MV_POSITIONS_START'] == _native.POSITIONS_START
    assert constants['MV_POSITIONS_END'] == _native.POSITIONS_END
    assert constants['MV_FLAG_FORCE_SIMT'] == _native.FLAG_FORCE_SIMT
    assert constants['MV_FLAG_PERSISTENT'] == _native.FLAG_PERSISTENT
    assert constants['MV_FLAG_FUSED_MERGE'] == _native.FLAG_FUSED_MERGE
    assert constants['MV_PATH_SIMT'] == _native.PATH_SIMT
    assert constants['MV_PATH_TMA_MMA'] == _native.PATH_TMA_MMA
    assert constants['MV_PATH_TMA_MMA_PERSISTENT'] == _native.PATH_TMA_MMA_PERSISTENT
    assert constants['MV_PATH_TMA_MMA_CLUSTER'] == _native.PATH_TMA_MMA_CLUSTER
    assert constants['MV_FLAG_CLUSTER'] == _native.FLAG_CLUSTER
    assert constants['MV_FLAG_WIDE'] == _native.FLAG_WIDE
    assert constants['MV_FLAG_CHUNK_ROWS'] == _native.FLAG_CHUNK_ROWS
    assert constants['MV_FLAG_CHUNK_MMA_SYNC'] == _native.FLAG_CHUNK_MMA_SYNC
    assert constants['MV_FLAG_CUDA_CORE_MATH'] == _native.FLAG_CUDA_CORE_MATH
    assert constants['MV_DEVICE_STATUS_WAIT_TIMEOUT'] == _native.DEVICE_STATUS_WAIT_TIMEOUT
    assert constants['MV_DEVICE_STATUS_BAD_PAGE_ID'] == _native.DEVICE_STATUS_BAD_PAGE_ID
    assert constants['MV_ABI_VERSION'] == _native.MV_ABI_VERSION


def test_argument_errors_are_reported_without_a_gpu():
    """Argument checks run before any CUDA call, so they work on a CPU host."""
    lib = _library()
    size = ctypes.c_size_t()
    status = lib.mv_paged_decode_workspace_size(4, 14, 3, 64, 16, 512, 0, 0, 2, ctypes.byref(size))
    assert status == 1
    assert b'divisible' in lib.mv_last_error()
    status = lib.mv_paged_decode(None, 0, 0, None, None, 1, 2, 16, 64, None, 0, 0, 1, None, 0, 16,
                                 1, 14, 0.125, None, 0, 0, None, 0, 0, 0, 2, None)
    assert status == 1
    assert b'must not be NULL' in lib.mv_last_error()
    status = lib.mv_write_paged_kv(None, 0, 0, 0, None, 0, 0, 0, None, None, 1, 1, 16, 64, None, 0,
                                   0, 1, None, 0, 0, 0, 1, 1, 2, None)
    assert status == 1


def test_status_errors_raise_native_error():
    from micro_vllm_b200 import _native
    _library()
    with pytest.raises(_native.NativeError, match='invalid argument'):
        _native.call('mv_paged_decode_workspace_size', 0, 1, 1, 1, 1, 1, 0, 0, 0,
                     ctypes.byref(ctypes.c_size_t()))


def test_import_loads_no_native_code():
    import subprocess
    import sys
    code = ('import sys; sys.path.insert(0, "micro-vllm_b200"); '
            'from micro_vllm_b200 import cuda_attention, cuda_paged_cache, _native; '
            'assert _native.library.cache_info().currsize == 0; '
            'assert cuda_attention._load_extension.cache_info().currsize == 0; '
            'assert cuda_paged_cache._load_extension.cache_info().currsize == 0')
    run = subprocess.run([sys.executable, '-c', code], cwd=ROOT, capture_output=True, text=True,
                         timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    from micro_vllm_b200 import _native
    monkeypatch.setattr(_native, 'LIB_PATH', tmp_path / 'absent.so')
    _native.library.cache_clear()
    try:
        with pytest.raises(RuntimeError, match='not built'):
            _native.library()
    finally:
        _native.library.cache_clear()
