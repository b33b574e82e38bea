import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN_PATH = ROOT / "tests" / "golden" / "reference_goldens.json"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def goldens():
    return json.loads(GOLDEN_PATH.read_text())


@pytest.fixture(scope="session")
def tiny(goldens):
    t = goldens["tiny_nnue"]
    return tuple(t["shape"]), {k: np.asarray(v, np.float32) for k, v in t["weights"].items()}


@pytest.fixture(scope="session")
def lib():
    import bulletou_b200

    return bulletou_b200.library()


@pytest.fixture(scope="session")
def ref_lib():
    import bulletou_b200

    try:
        return bulletou_b200.reference_library()
    except FileNotFoundError as e:  # built by oracle/build_ref.sh where the reference sources exist
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def ctx(lib):
    import bulletou_b200

    c = bulletou_b200.Context(0, lib)
    yield c
    c.close()


@pytest.fixture(scope="session")
def ref_ctx(ref_lib):
    import bulletou_b200

    c = bulletou_b200.Context(0, ref_lib)
    yield c
    c.close()


def assert_close(actual, expected, rtol, atol=0.0, name=""):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, f"{name}: shape {a.shape} != {e.shape}"
    if a.size == 0:
        return
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e)
    bad = np.nonzero(err > bound)[0] if a.ndim == 1 else np.argwhere(err > bound)
    assert bad.size == 0, (f"{name}: {bad.size} of {a.size} values out of tolerance "
                           f"(rtol={rtol}, atol={atol}); first at {bad[:5]}: "
                           f"actual={a.reshape(-1)[bad[:5]] if a.ndim == 1 else None} "
                           f"expected={e.reshape(-1)[bad[:5]] if a.ndim == 1 else None}, max err {err.max():.3e}")


def assert_close_scaled(actual, expected, rel, name=""):
    """|a - e| <= rel * max|e| (tolerance relative to the tensor's scale, for
    sums whose summation order differs)."""
    e = np.asarray(expected, np.float64)
    scale = max(float(np.abs(e).max()) if e.size else 0.0, 1e-30)
    assert_close(actual, expected, 0.0, rel * scale, name)
