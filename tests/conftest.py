import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


@pytest.fixture(autouse=True)
def _cuda_math_for_gpu_tests(request):
    """GPU tests compare kernels with the oracle byte for byte, so inside them
    the oracle takes CUDA's own rsqrtf / expf values (evaluated on the GPU by
    oracle/_ref/libqo_gpu_checks.so); CPU tests keep the correctly rounded
    host stand-ins."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    import torch

    if not torch.cuda.is_available():
        yield
        return
    from oracle import cuda_math, producers

    with producers.use_math(cuda_math.CudaMath()):
        yield
