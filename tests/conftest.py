import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / 'tests' / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


@pytest.fixture(scope='session')
def golden():
    import numpy as np

    def load(name):
        return dict(np.load(GOLDEN / f'{name}.npz', allow_pickle=False))

    return load


@pytest.fixture(scope='session')
def digests():
    import json
    return json.loads((GOLDEN / 'digests.json').read_text())


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip('CUDA device required')
    from bevfusion_triton_b200 import load_native
    load_native()
    return torch.device('cuda:0')
