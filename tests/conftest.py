import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def engine_factory():
    """Engines are cached per shape so a test session creates few handles."""
    from whallm_b200.moe import Engine
    cache = {}

    def make(max_tokens, hidden, inter, experts, topk, gemv_max_tokens=0):
        key = (max_tokens, hidden, inter, experts, topk, gemv_max_tokens)
        if key not in cache:
            cache[key] = Engine(0, max_tokens=max_tokens, hidden=hidden, inter=inter, experts=experts, topk=topk,
                                gemv_max_tokens=gemv_max_tokens)
        return cache[key]

    yield make
    for eng in cache.values():
        eng.ctx.close()
