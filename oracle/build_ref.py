"""Build recipe for the reference's own CUDA extensions (a comparison checker).

Compiles, from the sources where they lie in the reference tree, the two
torch extensions the reference JIT-loads for the hot path:

* ``_micro_vllm_decode_attention`` -- src/micro_vllm/csrc/decode_attention.cpp,
  decode_attention.cu, decode_attention_online.cu, decode_attention_paged.cu
  (loaded by src/micro_vllm/cuda_attention.py:9-23), whose
  ``_decode_attention_paged`` is the reference's paged decode kernel;
* ``_micro_vllm_paged_cache`` -- src/micro_vllm/csrc/paged_kv_cache.cpp and
  paged_kv_cache.cu (loaded by src/micro_vllm/cuda_paged_cache.py:9-20).

The compiler is driven directly (nvcc for .cu, g++ for .cpp, the flags torch's
extension builder would pass, -O2 as the reference asks, sm_100a), not through
the reference's loader. Outputs go to oracle/_ref/ only (git-ignored; they
travel with the repository to the GPU machine, where the reference tree is
absent). Test infrastructure: only GPU tests load these modules, to compare
this library's kernels with the reference's own on the same inputs.

Usage: python oracle/build_ref.py REFERENCE_ROOT  (or set MICRO_VLLM_REFERENCE_ROOT)
"""
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

OUT_DIR = Path(__file__).resolve().parent / '_ref'

EXTENSIONS = {
    '_micro_vllm_decode_attention': ('decode_attention.cpp', 'decode_attention.cu',
                                     'decode_attention_online.cu', 'decode_attention_paged.cu'),
    '_micro_vllm_paged_cache': ('paged_kv_cache.cpp', 'paged_kv_cache.cu'),
}


def _torch_flags():
    import torch
    from torch.utils import cpp_extension
    includes = [*cpp_extension.include_paths(), sysconfig.get_paths()['include']]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defines = ['-DTORCH_API_INCLUDE_EXTENSION_H', f'-D_GLIBCXX_USE_CXX11_ABI={abi}']
    libs = cpp_extension.library_paths()
    return includes, defines, libs


def _run(cmd):
    subprocess.run(cmd, check=True)


def build(reference_root, force=False):
    """Build both extensions into oracle/_ref; returns the module paths built.

    Skips (returns []) when the reference tree is absent, as on the GPU
    machine, where the modules built here are used as they are.
    """
    csrc = Path(reference_root) / 'src' / 'micro_vllm' / 'csrc'
    if not csrc.is_dir():
        return []
    nvcc = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    cuda_home = Path(nvcc).resolve().parent.parent
    includes, defines, libs = _torch_flags()
    inc = [f'-I{p}' for p in includes]
    OUT_DIR.mkdir(exist_ok=True)
    built = []
    for name, sources in EXTENSIONS.items():
        target = OUT_DIR / f'{name}.so'
        newest = max((csrc / s).stat().st_mtime for s in sources)
        if target.exists() and not force and target.stat().st_mtime >= newest:
            built.append(target)
            continue
        objects = []
        for source in sources:
            src = csrc / source
            obj = OUT_DIR / f'{name}.{source}.o'
            common = [*inc, *defines, f'-DTORCH_EXTENSION_NAME={name}', '-O2', '-std=c++17']
            if source.endswith('.cu'):
                _run([nvcc, '-c', str(src), '-o', str(obj), *common,
                      '-gencode', 'arch=compute_100a,code=sm_100a',
                      '-D__CUDA_NO_HALF_OPERATORS__', '-D__CUDA_NO_HALF_CONVERSIONS__',
                      '-D__CUDA_NO_BFLOAT16_CONVERSIONS__', '-D__CUDA_NO_HALF2_OPERATORS__',
                      '--expt-relaxed-constexpr', '-Xcompiler', '-fPIC'])
            else:
                _run(['g++', '-c', str(src), '-o', str(obj), *common, '-fPIC',
                      f'-I{cuda_home / "include"}'])
            objects.append(str(obj))
        tmp = OUT_DIR / f'.{name}.so.tmp'
        _run(['g++', '-shared', *objects, '-o', str(tmp),
              *[f'-L{p}' for p in libs], *[f'-Wl,-rpath,{p}' for p in libs],
              f'-L{cuda_home / "lib64"}', '-lc10', '-lc10_cuda', '-ltorch', '-ltorch_cpu', '-ltorch_cuda',
              '-ltorch_python', '-lcudart'])
        os.replace(tmp, target)
        for obj in objects:
            Path(obj).unlink()
        built.append(target)
    return built


def load(name):
    """Import a built extension module from oracle/_ref (None if it is absent)."""
    import importlib.machinery
    import importlib.util
    path = OUT_DIR / f'{name}.so'
    if not path.exists():
        return None
    import torch  # noqa: F401  (the module links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


if __name__ == '__main__':
    source = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('MICRO_VLLM_REFERENCE_ROOT')
    if not source:
        raise SystemExit('usage: python oracle/build_ref.py REFERENCE_ROOT')
    for path in build(Path(source), force=True):
        print(path)
