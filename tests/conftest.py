import itertools
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def golden_dir():
    return GOLDEN


@pytest.fixture
def seq_block_size():
    """Temporarily sets Sequence.block_size and resets the id counter (the reference tests'
    autouse fixture, tests/test_correctness.py:10-18)."""
    from hilda_vllm_b200.engine.sequence import Sequence

    orig_bs, orig_counter = Sequence.block_size, Sequence.counter

    def set_bs(bs):
        Sequence.block_size = bs
        Sequence.counter = itertools.count()

    yield set_bs
    Sequence.block_size, Sequence.counter = orig_bs, orig_counter
