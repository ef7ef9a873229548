"""Build libmvdecode.so in-tree for sm_100a with nvcc.

    python -m micro_vllm_b200.build        (from the micro-vllm_b200/ source root)

The library links the CUDA runtime statically and resolves the driver's
tensor-map encoder at run time, so it needs only the NVIDIA driver next to it.
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC_DIR = PACKAGE_DIR / 'csrc'
LIB_DIR = PACKAGE_DIR / 'lib'
LIB_PATH = LIB_DIR / 'libmvdecode.so'
INCLUDE_DIR = PACKAGE_DIR.parents[1] / 'include'

NVCC_FLAGS = [
    '-gencode', 'arch=compute_100a,code=sm_100a',
    '-lineinfo', '-O3', '-std=c++17',
    '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
    '-shared',
]


def nvcc_path() -> str:
    found = shutil.which('nvcc')
    if found:
        return found
    cuda_home = os.environ.get('CUDA_HOME', '/usr/local/cuda')
    return str(Path(cuda_home) / 'bin' / 'nvcc')


def sources():
    return sorted(CSRC_DIR.glob('*.cu')) + sorted(CSRC_DIR.glob('*.cuh'))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    inputs = list(sources()) + [INCLUDE_DIR / 'mvdecode.h', Path(__file__)]
    return any(path.stat().st_mtime > built for path in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library unless it is newer than every source; return its path."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix('.so.tmp')
    cmd = [nvcc_path(), *NVCC_FLAGS, '-I', str(INCLUDE_DIR), '-o', str(tmp),
           str(CSRC_DIR / 'mv_capi.cu')]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
        print(' '.join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
