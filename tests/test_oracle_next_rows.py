"""Oracles of the "next" rows the reference does not have: the fused residual
add (pinned to torch's own ``x + r`` in x's dtype on CPU, the norm to the torch
port of the reference's AllReduce path applied to z) and the backward pass
(pinned to torch autograd of that port, in float64)."""
import numpy as np
import pytest
import torch

from gpu_helpers import NAMES, to_np
from oracle import tp_rmsnorm as O
from oracle import torch_port
from rmsnorm_tp_b200.workloads import make_group


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tp,rows,hidden", [(1, 7, 96), (2, 16, 256), (4, 5, 512), (8, 3, 1024)])
def test_residual_oracle_matches_torch(dtype, tp, rows, hidden):
    name = NAMES[dtype]
    xs, ws = make_group(rows, hidden, tp, dtype, 300)
    rs, _ = make_group(rows, hidden, tp, dtype, 400)
    zs_t = [x + r for x, r in zip(xs, rs)]                       # torch, x's dtype
    ys_t = torch_port.allreduce_path_group(zs_t, ws, 1e-6)
    ys, zs = O.allreduce_path_residual([to_np(x) for x in xs], [to_np(r) for r in rs],
                                       [to_np(w) for w in ws], 1e-6, name)
    for z, zt in zip(zs, zs_t):
        assert np.array_equal(np.asarray(z), to_np(zt))          # bit-exact add
    for y, yt in zip(ys, ys_t):
        got = O.round_to(name, y)
        want = O.round_to(name, yt.float().numpy())
        assert O.compare(name, got, want)["ok"]
    # the fused formula on z stays within the parity tolerance of the AllReduce path
    yf, zf = O.fused_path_residual([to_np(x) for x in xs], [to_np(r) for r in rs],
                                   [to_np(w) for w in ws], 1e-6, name)
    for a, b in zip(zf, zs):
        assert np.array_equal(np.asarray(a), np.asarray(b))
    for a, b in zip(yf, ys):
        assert O.compare(name, O.round_to(name, a), O.round_to(name, b))["ok"]


def test_residual_oracle_catches_an_unrounded_add():
    """A planted mistake: z kept in fp32 instead of rounded to bf16 changes the
    updated residual, which the bit-exact check of z catches."""
    xs, _ = make_group(64, 512, 1, torch.bfloat16, 5)
    rs, _ = make_group(64, 512, 1, torch.bfloat16, 6)
    x, r = to_np(xs[0]), to_np(rs[0])
    good = O.residual_add(x, r, "bf16")
    planted = O.to_f32("bf16", x) + O.to_f32("bf16", r)          # no rounding
    assert not np.array_equal(O.to_f32("bf16", good), planted)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tp,rows,hidden", [(1, 7, 96), (2, 16, 256), (4, 5, 512), (8, 3, 1024)])
def test_backward_oracle_matches_autograd_of_the_reference_formula(dtype, tp, rows, hidden):
    """The backward oracle (closed form) against torch autograd, in float64, of the
    torch port of the reference's AllReduce path (bench_rmsnorm_tp.py:16-22)."""
    name = NAMES[dtype]
    xs, ws = make_group(rows, hidden, tp, dtype, 500)
    dys, _ = make_group(rows, hidden, tp, dtype, 600)
    x64 = [x.double().requires_grad_() for x in xs]
    w64 = [w.double().requires_grad_() for w in ws]
    ys = torch_port.allreduce_path_group(x64, w64, 1e-6)
    sum((y * dy.double()).sum() for y, dy in zip(ys, dys)).backward()
    dxs, dws = O.backward_path([to_np(x) for x in xs], [to_np(d) for d in dys],
                               [to_np(w) for w in ws], 1e-6, name)
    for dx, dw, xt, wt in zip(dxs, dws, x64, w64):
        np.testing.assert_allclose(dx, xt.grad.numpy(), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(dw, wt.grad.numpy(), rtol=1e-5, atol=1e-6)


def test_dw_tolerance_covers_fp32_two_level_summation():
    """The dw tolerance is justified by an fp32 emulation of the kernels' own
    summation order (per-CTA partials over rows c, c + 296, ..., then the 296
    partials in order) at 2500 rows of width 2048: within the accumulation-aware
    tolerance with a wide margin, while a tolerance relative to |dw| alone would
    reject it (|dw| can be far below the magnitude of its terms)."""
    rows, hidden, grid = 2500, 2048, 296
    xs, ws = make_group(rows, hidden, 1, torch.float32, 13)
    dys, _ = make_group(rows, hidden, 1, torch.float32, 104)
    x, dy = xs[0].numpy(), dys[0].numpy()
    want = O.backward_path([x], [dy], [ws[0].numpy()], 1e-6, "f32")[1][0]
    scale = O.dw_magnitude([x], [dy], 1e-6, "f32")[0]
    S = (x * x).sum(axis=1, dtype=np.float32)
    inv = (1.0 / np.sqrt(S / np.float32(hidden) + np.float32(1e-6))).astype(np.float32)
    parts = np.zeros((grid, hidden), np.float32)
    for c in range(grid):
        for r in range(c, rows, grid):
            parts[c] += (dy[r] * x[r]) * inv[r]
    got = np.zeros(hidden, np.float32)
    for c in range(grid):
        got += parts[c]
    assert O.compare_backward("f32", got, want, scale)["ok"]
    diff = np.abs(got.astype(np.float64) - want)
    margin = (np.maximum(1e-5, 32 * O.FP32_UNIT * scale) + 1e-4 * np.abs(want)) / np.maximum(diff, 1e-30)
    assert margin.min() > 10
    assert not O.compare_backward("f32", got, want)["ok"]      # |dw|-relative only: too tight
