"""Import the unmodified micro-vllm reference installed in baseline/_ref.

``baseline/install_ref.py`` installs it (git-ignored; the directory travels
with the working tree to the GPU machine). Tests use the reference's own
modules -- its ``PagedKVCache``, model code and CPU attention -- and route its
native names to this package with ``micro_vllm_b200.integration``.
"""
import importlib
import sys
from pathlib import Path

import pytest

REF_DIR = Path(__file__).resolve().parents[1] / 'baseline' / '_ref'


def available() -> bool:
    return (REF_DIR / 'micro_vllm' / '__init__.py').is_file()


def reference(module='micro_vllm'):
    """Import ``module`` from the installed reference; fail the test if it is not installed."""
    if not available():
        pytest.fail('micro-vllm is not installed in baseline/_ref: run '
                    'python baseline/install_ref.py REFERENCE_ROOT')
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    return importlib.import_module(module)
