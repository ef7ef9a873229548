"""Install the unmodified micro-vllm reference into baseline/_ref (git-ignored).

Usage: python baseline/install_ref.py REFERENCE_ROOT
       (or set MICRO_VLLM_REFERENCE_ROOT)

Runs ``pip install --no-index --no-build-isolation --no-deps --target
baseline/_ref`` on a temporary copy of the reference tree (the tree itself may
be read-only and setuptools writes build files next to the sources). torch and
transformers, micro-vllm's only dependencies, are already in the environment,
hence ``--no-deps``. The installed package is micro-vllm's pure-Python code
plus its csrc sources as package data; nothing is compiled (its CUDA
extensions are JIT-built only when first called, and the tests and the bench
never call them through this install -- oracle/build_ref.py builds them).

baseline/_ref travels with the working tree to the GPU machine, where the
reference tree is absent. Used by: the tests that run the reference's own
model code and ``PagedKVCache`` on this package's kernels, and ``bench.py
--impl reference`` (the reference's CPU path timed on the host cores).
"""
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

TARGET = Path(__file__).resolve().parent / '_ref'


def install(reference_root, force=False):
    """Install into baseline/_ref; returns the target path (unchanged if present and not forced)."""
    root = Path(reference_root)
    if not (root / 'pyproject.toml').is_file() or not (root / 'src' / 'micro_vllm').is_dir():
        raise FileNotFoundError(f'{root} is not a micro-vllm checkout')
    if (TARGET / 'micro_vllm' / '__init__.py').is_file() and not force:
        return TARGET
    with tempfile.TemporaryDirectory(prefix='mvref_') as scratch:
        copy = Path(scratch) / 'src_tree'
        shutil.copytree(root, copy, ignore=shutil.ignore_patterns('__pycache__', '*.pyc', '.git'))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, '-m', 'pip', 'install', '--no-index', '--no-build-isolation', '--no-deps',
               '--quiet', '--target', str(TARGET), str(copy)]
        wheelhouse = Path('/opt/wheelhouse')
        if wheelhouse.is_dir():
            cmd[4:4] = ['--find-links', str(wheelhouse)]
        subprocess.run(cmd, check=True, env=dict(os.environ, PYTHONDONTWRITEBYTECODE='1'))
    return TARGET


if __name__ == '__main__':
    source = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('MICRO_VLLM_REFERENCE_ROOT')
    if not source:
        raise SystemExit('usage: python baseline/install_ref.py REFERENCE_ROOT')
    print(install(source, force=True))
