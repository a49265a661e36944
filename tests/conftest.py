import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a B200)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN / "golden_small.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def config1():
    with np.load(GOLDEN / "config1.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def gptq_golden():
    with np.load(GOLDEN / "gptq_small.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def qcol_golden():
    with np.load(GOLDEN / "quantize_col.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def gptq_ao_golden():
    with np.load(GOLDEN / "gptq_act_order.npz") as z:
        return {k: z[k] for k in z.files}


def golden_values(arr: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 values of a golden array stored by make_golden._np (bf16 as uint16 bits)."""
    if dtype == "bfloat16":
        return (arr.astype(np.uint32) << 16).view(np.float32)
    return arr.astype(np.float32)


SHORT = {"float16": "f16", "bfloat16": "bf16", "float32": "f32"}
