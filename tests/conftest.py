import os
import sys

import pytest

# every core mutex acquisition is checked against the lock hierarchy in tests
os.environ.setdefault("KVBM_LOCK_CHECK", "1")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2+ CUDA GPUs")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        have_gpu = torch.cuda.is_available()
        ngpu = torch.cuda.device_count() if have_gpu else 0
    except Exception:  # pragma: no cover
        have_gpu, ngpu = False, 0
    skip_gpu = pytest.mark.skip(reason="no CUDA GPU")
    skip_multi = pytest.mark.skip(reason="needs 2+ GPUs")
    for item in items:
        if "gpu" in item.keywords and not have_gpu:
            item.add_marker(skip_gpu)
        if "multigpu" in item.keywords and ngpu < 2:
            item.add_marker(skip_multi)
