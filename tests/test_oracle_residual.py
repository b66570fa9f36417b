"""Oracle of the fused residual add (a "next" row: the reference has no
residual). The add is pinned to torch's own ``x + r`` in x's dtype on CPU, and
the norm to the torch port of the reference's AllReduce path applied to z."""
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
