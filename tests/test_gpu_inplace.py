"""out may alias x (in place): the kernels never read an element of x after
writing the same element of the output. Checked for the local, register, bulk and
generic kernels, the emulated group and the fused residual add."""
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,hidden", [(300, 4096), (65536, 4096), (50, 37)])
def test_local_in_place(family, rows, hidden):
    xs, ws = make_group(rows, hidden, 1, torch.bfloat16, 61, device="cuda")
    want = rtp.local_rmsnorm(xs[0], ws[0], 1e-6)
    x = xs[0].clone()
    r = xs[0].flip(0).contiguous()
    want_res = rtp.local_rmsnorm(xs[0], ws[0], 1e-6, residual=r.clone())
    got = rtp.local_rmsnorm(x, ws[0], 1e-6, out=x)
    torch.cuda.synchronize()
    assert got.data_ptr() == x.data_ptr() and torch.equal(x, want)
    x = xs[0].clone()
    rtp.local_rmsnorm(x, ws[0], 1e-6, out=x, residual=r)
    torch.cuda.synchronize()
    assert torch.equal(x, want_res)


def test_emulated_group_in_place():
    xs, ws = make_group(200, 2 * 1024, 2, torch.bfloat16, 62, device="cuda")
    g = rtp.EmulatedTPGroup(2, eps=1e-6, num_max_rows=256, timeout_s=5.0)
    try:
        want = g.forward(xs, ws)
        xc = [x.clone() for x in xs]
        g.forward(xc, ws, outs=xc)
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(xc, want))
    finally:
        g.destroy()
