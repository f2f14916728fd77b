import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "gpu-sparse_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size configuration")
    config.addinivalue_line("markers", "tensorcore: runs the head terms on the tensor cores "
                                       "(checked within the 1e-5 tolerance, not bit for bit)")


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


@pytest.fixture(autouse=True)
def head_mode(request):
    """Bit-exact tests run the head terms in the canonical CUDA-core order (the oracle's);
    tests marked ``tensorcore`` force the tensor-core head phase.  The library's default
    (automatic) mode is restored afterwards."""
    try:
        import gpusparse._lib as L
        lib = L.lib()
    except Exception:          # no library: nothing to set (CPU-only checks)
        yield
        return
    mode = L.HEAD_TENSOR_CORES if request.node.get_closest_marker("tensorcore") else L.HEAD_CUDA_CORES
    L.check(lib.gsp_set_head_mode(mode), "head mode")
    try:
        yield
    finally:
        lib.gsp_set_head_mode(L.HEAD_AUTO)
