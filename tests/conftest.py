import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "yolo-baremetal_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def gpu_present() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def workdir(tmp_path_factory):
    return tmp_path_factory.mktemp("yb")


@pytest.fixture(scope="session")
def weights_n0(workdir):
    """YOLO26n random-init weights, seed 0 (the benchmark's recipe)."""
    import yb_weights as yw

    path = str(workdir / "yolo26n_seed0.bin")
    yw.write_bin(path, yw.random_state("n", 0))
    return path


@pytest.fixture(scope="session")
def weights_n0_soft(workdir):
    """Seed-0 weights with the final class convs scaled by 0.01: scores stay
    below sigmoid saturation, so the top-k order is decided by scores."""
    import yb_weights as yw

    path = str(workdir / "yolo26n_seed0_soft.bin")
    yw.write_bin(path, yw.random_state("n", 0, cls_scale=0.01))
    return path


@pytest.fixture(scope="session")
def weights_n0_o2m(workdir):
    """Seed-0 weights (class convs scaled by 0.01, so scores rank) with the
    one-to-one Detect branches removed: only model.23.cv2 / model.23.cv3
    remain, which the reference falls back to (detect.c:297-299)."""
    import yb_weights as yw

    path = str(workdir / "yolo26n_seed0_o2m.bin")
    sd = yw.random_state("n", 0, cls_scale=0.01)
    yw.write_bin(path, type(sd)((k, v) for k, v in sd.items() if ".one2one_" not in k))
    return path


@pytest.fixture(scope="session")
def weights_s0(workdir):
    import yb_weights as yw

    path = str(workdir / "yolo26s_seed0.bin")
    yw.write_bin(path, yw.random_state("s", 0))
    return path


def golden(name: str):
    import yb_weights as yw

    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.fail(f"golden fixture {name} is missing from tests/golden")
    return yw.read_records(path)


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0
