import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def load_golden():
    """{case: {"meta": dict, "x": [..], "w": [..], "y": [..]}} from tests/golden/golden.npz."""
    cases = {}
    with np.load(GOLDEN) as z:
        names = sorted({k.split("/")[0] for k in z.files})
        for n in names:
            meta = json.loads(bytes(z[f"{n}/meta"]).decode())
            tp = meta["tp"]
            cases[n] = {
                "meta": meta,
                "x": [z[f"{n}/x{r}"] for r in range(tp)],
                "w": [z[f"{n}/w{r}"] for r in range(tp)],
                "y": [z[f"{n}/y{r}"] for r in range(tp)],
            }
    return cases


@pytest.fixture(scope="session")
def golden():
    return load_golden()


@pytest.fixture(autouse=True)
def _require_cuda_for_gpu_tests(request):
    # A GPU test must never pass by skipping on a box without CUDA.
    if request.node.get_closest_marker("gpu") is not None:
        import torch

        assert torch.cuda.is_available(), "GPU test run without a CUDA device"


@pytest.fixture(params=["auto", "bulk", "register", "batch"])
def family(request):
    """Run a test once per kernel family: the automatic choice (which includes the
    resident register kernels with an exchange), bulk-copy, rotating register and
    batch kernels."""
    import rmsnorm_tp_b200 as rtp

    rtp.set_kernel_family(request.param)
    yield request.param
    rtp.set_kernel_family("auto")
