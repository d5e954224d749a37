import os
import sys

# separate hardware queues for the library's concurrent streams (read when the CUDA context
# is created, so it is set before anything can create one; the package sets the same default)
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

import pytest  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def ref_root():
    """Directory holding the unmodified reference package (``femtotron``), installed into
    baseline/_ref on first use.  A test that needs it fails, rather than skips, when the
    reference cannot be installed."""
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    try:
        import install_reference
    finally:
        sys.path.pop(0)
    if not install_reference.installed():
        install_reference.install()
    return install_reference.TARGET
