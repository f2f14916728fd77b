import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "gpu-sparse_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size configuration")


import pytest  # noqa: E402


@pytest.fixture
def shared_buffers_only():
    """Score through the shared candidate buffers even for small batches (the tests of
    the buffer protocol, its bounded waits and the shared bound between shards), then
    restore the small-batch mode's limit."""
    import gpusparse._lib as L
    lib = L.lib()
    default = lib.gsp_get_tree_limit()
    L.check(lib.gsp_set_tree_limit(0), "tree limit")
    try:
        yield
    finally:
        lib.gsp_set_tree_limit(default)
