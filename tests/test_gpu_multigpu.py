"""Real multi-GPU group (CUDA IPC over NVLink, NCCL bootstrap): runs
tests/mp_tp_worker.py (and, on 8 GPUs, a shortened tests/mp_stress_worker.py)
under torchrun on 2 or more GPUs, as child processes, with NVLS off (a rank that
leaves a test must not hold multicast memory)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("nproc", [2, 4, 8])
def test_real_group_over_nvlink(nproc):
    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs, have {torch.cuda.device_count()}")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", RMSNORM_TP_TIMEOUT_MS="10000")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "mp_tp_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    tail = (res.stdout[-3000:] + "\n" + res.stderr[-3000:])
    assert res.returncode == 0, tail
    assert "ALL OK" in res.stdout, tail


def test_stress_config_real_group_of_8():
    """The stress configuration (hidden 16384, 65536 rows, outliers, zero rows)
    across the 32-bit tag wrap with random per-rank skew; 2 x 10^4 calls here
    (the full 10^5-call run is the worker's default)."""
    if torch.cuda.device_count() < 8:
        pytest.skip(f"needs 8 GPUs, have {torch.cuda.device_count()}")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=8", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "mp_stress_worker.py"), "--calls", "20000",
           "--check-every", "5000"]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    tail = (res.stdout[-3000:] + "\n" + res.stderr[-3000:])
    assert res.returncode == 0, tail
    assert "STRESS OK" in res.stdout, tail
