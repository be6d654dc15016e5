import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qx-mini-c_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

# The reference source tree (read-only); only the checker build and the
# fixture generator use it.
REFERENCE_TREE = os.environ.get("QX_REFERENCE_TREE", "/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA engine)")


@pytest.fixture(scope="session")
def mini_image():
    import qxlib
    return qxlib.build_image(qxlib.mini_config(7))


@pytest.fixture(scope="session")
def full_image():
    """The full-size seeded Qwen3-30B-A3B synthetic model (about 10.25 GB)."""
    import qxlib
    return qxlib.build_image(qxlib.synth_config(7))


@pytest.fixture(scope="session")
def port():
    import oracle_bind
    c = oracle_bind.Checker("port")
    c.lib.qxo_set_threads(os.cpu_count() or 1)
    return c


@pytest.fixture(scope="session")
def ref():
    import oracle_bind
    if not oracle_bind.available("ref"):
        pytest.skip("reference checker not built (needs the reference tree)")
    return oracle_bind.Checker("ref")
