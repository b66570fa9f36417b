"""Oracle of the fused row-parallel linear -> reduce-scatter -> TP RMSNorm
(oracle/tp_rmsnorm.py linear_rs_norm_path), pinned against the same pipeline in
torch ops (oracle/torch_port.py linear_rs_norm_group: fp32 GEMM, the partial
rounded to the dtype, rank-order sum per column block, the reference's
AllReduce norm), and the C-ABI checks of its entry points (no GPU)."""
import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import NAMES, to_np
from oracle import tp_rmsnorm as O
from oracle import torch_port
from rmsnorm_tp_b200 import _lib
from rmsnorm_tp_b200.workloads import make_group, make_linear_group


@pytest.mark.parametrize("tp", [1, 2, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("rows,k,hidden", [(5, 64, 256), (33, 128, 512)])
def test_linear_oracle_matches_torch_pipeline(tp, dtype, residual, rows, k, hidden):
    name = NAMES[dtype]
    as_, lws, gs = make_linear_group(rows, k, hidden * tp // tp, tp, dtype, 10 + rows)
    rs = make_group(rows, hidden, tp, dtype, 20 + rows)[0] if residual else None
    want_t = torch_port.linear_rs_norm_group(as_, lws, gs, 1e-5, rs)
    got, zs = O.linear_rs_norm_path([to_np(a) for a in as_], [to_np(w) for w in lws],
                                    [to_np(g) for g in gs], 1e-5, name,
                                    None if rs is None else [to_np(r) for r in rs])
    for r in range(tp):
        res = O.compare(name, O.round_to(name, got[r]),
                        O.round_to(name, want_t[r].float().numpy()))
        assert res["ok"], (r, res)
    # z is x (+ residual): rows of unit variance after the sum over ranks
    z = np.concatenate([O.to_f32(name, zz) for zz in zs], axis=1)
    assert 0.5 < float(z.std()) < (2.0 if not residual else 3.0)


def test_linear_reduce_scatter_sums_in_rank_order():
    # three partials whose fp32 sum depends on the order: rank order is the contract
    p0 = np.full((1, 2), 1.0, np.float32)
    p1 = np.full((1, 2), 2.0 ** 24, np.float32)
    p2 = np.full((1, 2), -(2.0 ** 24), np.float32)
    xs = O.linear_reduce_scatter([np.tile(p, (1, 3)) for p in (p0, p1, p2)], "f32")
    assert all(float(x[0, 0]) == 0.0 for x in xs)        # (1 + 2^24) - 2^24 = 0 in fp32


def test_create_linear_rejects_bad_arguments_before_touching_cuda():
    out = ctypes.c_void_p()
    L = _lib.LIB
    for tp, hidden in ((2, 100), (2, 128), (4, 256 * 3), (0, 1024), (9, 1024)):
        assert L.rmsnorm_tp_create_linear(0, tp, 64, hidden, 0, ctypes.byref(out)) == _lib.ERR_INVALID
        assert out.value is None
    assert "multiple of tp" in _lib.last_error() or "tp_size" in _lib.last_error()


def test_linear_forward_validates_without_gpu():
    L = _lib.LIB
    assert L.rmsnorm_tp_linear_forward(None, None, None, None, None, None, 4, 64, 1, 1e-6,
                                       None) == _lib.ERR_INVALID
    assert L.rmsnorm_tp_linear_forward_emulated(None, 2, None, None, None, None, None, 4, 64, 1,
                                                1e-6, None) == _lib.ERR_INVALID


def test_linear_tile_order_is_a_bijection(tmp_path):
    """tests/cpp/test_linear_tiles.cpp: the fused linear's tile order covers every
    output tile exactly once (compiled against the kernels' header)."""
    import os
    import subprocess

    from conftest import ROOT

    exe = tmp_path / "test_linear_tiles"
    subprocess.run(["g++", "-O2", "-std=c++17", "-Wall", "-I",
                    os.path.join(ROOT, "rmsnorm_tp_b200", "csrc"),
                    os.path.join(ROOT, "tests", "cpp", "test_linear_tiles.cpp"), "-o", str(exe)],
                   check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "ALL PASS" in res.stdout, res.stdout
