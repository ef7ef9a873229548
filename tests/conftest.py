import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / 'micro-vllm_b200'):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a)')
    config.addinivalue_line('markers', 'slow: full-size workload')


@pytest.fixture(scope='session')
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('GPU test selected but CUDA is not available')
    return torch.device('cuda', 0)
