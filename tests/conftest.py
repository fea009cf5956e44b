"""Test configuration: import path, markers, GPU auto-skip, RNG isolation, tolerances.

Tolerance policy (as in the reference suite): 0 where the reduction order is the
same, ~1e-6 for fp32 reductions in a different order, ~1e-5 after optimizer
steps; bf16 kernels are compared with an fp32 PyTorch statement of the same op
at bf16-appropriate tolerances.
"""

from __future__ import annotations

import os
import random
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
os.environ.setdefault("PYTHONPATH", str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

FP32_REORDER_ATOL = 1e-6
ADAM_ATOL = 1e-5


def pytest_configure(config: pytest.Config) -> None:
    for name, text in (("gpu", "needs a CUDA device (B200, sm_100a)"), ("multigpu", "needs two or more CUDA devices"),
                       ("distributed", "spawns several CPU/Gloo ranks"), ("slow", "long-running")):
        config.addinivalue_line("markers", f"{name}: {text}")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    gpus = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for item in items:
        if "gpu" in item.keywords and gpus == 0:
            item.add_marker(pytest.mark.skip(reason=f"needs a CUDA device; {gpus} visible"))
        if "multigpu" in item.keywords and gpus < 2:
            item.add_marker(pytest.mark.skip(reason=f"needs >= 2 CUDA devices; {gpus} visible"))


@pytest.fixture(autouse=True)
def _isolated_rng():
    state = (random.getstate(), np.random.get_state(), torch.get_rng_state())
    torch.manual_seed(0)
    yield
    random.setstate(state[0])
    np.random.set_state(state[1])
    torch.set_rng_state(state[2])
