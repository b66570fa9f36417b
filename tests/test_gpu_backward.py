"""GPU parity of the backward pass (dx, dw; through the C-ABI) against the
closed-form oracle (oracle.tp_rmsnorm.backward_path, itself pinned to torch
autograd of the reference's formula). TP = 1, emulated TP = 2/4/8, the real
entry point with host-written peer slots (both exchanges, two generations), the
generation sequence forward / backward / forward, autograd, and a bounded wait
that runs out. Tolerances: oracle.tp_rmsnorm.BACKWARD_TOLERANCE."""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import NAMES, check_against_oracle, device_view, out_f32, pack_slots, slot_index, to_np
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200 import _lib
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


def _inputs(rows, hidden, tp, dtype, seed):
    xs, ws = make_group(rows, hidden, tp, dtype, seed, device="cuda")
    dys, _ = make_group(rows, hidden, tp, dtype, seed + 91, device="cuda")
    return xs, ws, dys


def _check(dtype, xs, ws, dys, dxs, dws, eps):
    name = NAMES[dtype]
    want_dx, want_dw = O.backward_path([to_np(x) for x in xs], [to_np(d) for d in dys],
                                       [to_np(w) for w in ws], eps, name)
    scale = O.dw_magnitude([to_np(x) for x in xs], [to_np(d) for d in dys], eps, name)
    for k in range(len(xs)):
        r = O.compare_backward(name, out_f32(name, dxs[k]), O.round_to(name, want_dx[k]))
        assert r["ok"], f"dx rank {k}: {r}"
        r = O.compare_backward(name, out_f32(name, dws[k]), O.round_to(name, want_dw[k]), scale[k])
        assert r["ok"], f"dw rank {k}: {r}"


@pytest.fixture(params=["auto", "bulk"])
def bwd_family(request):
    """The register backward kernel (automatic choice for aligned rows) and the
    one-CTA-per-row kernel (kept under the bulk family)."""
    rtp.set_kernel_family(request.param)
    yield request.param
    rtp.set_kernel_family("auto")


@pytest.fixture(params=["auto", "register", "bulk"])
def local_bwd_family(request):
    """TP = 1: the ring kernel (automatic choice for aligned rows: bulk copies of
    x and dy into shared memory), the double-buffered register kernel (register
    family) and the one-CTA-per-row kernel (bulk family)."""
    rtp.set_kernel_family(request.param)
    yield request.param
    rtp.set_kernel_family("auto")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hidden", [37, 96, 512, 4096, 8192, 16384])
@pytest.mark.parametrize("rows", [1, 7, 300, 2500])
def test_local_backward(local_bwd_family, dtype, hidden, rows):
    xs, ws, dys = _inputs(rows, hidden, 1, dtype, 13)
    dx, dw = rtp.local_rmsnorm_backward(dys[0], xs[0], ws[0], 1e-6)
    torch.cuda.synchronize()
    _check(dtype, xs, ws, dys, [dx], [dw], 1e-6)
    dx2, dw2 = rtp.local_rmsnorm_backward(dys[0], xs[0], ws[0], 1e-6)   # deterministic
    torch.cuda.synchronize()
    assert torch.equal(dx, dx2) and torch.equal(dw, dw2)


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hl,rows", [(64, 5), (512, 300), (2048, 1), (37, 40), (1024, 129)])
def test_emulated_group_backward_between_forwards(bwd_family, tp, dtype, hl, rows):
    """forward, backward, forward on one group: the backward takes two
    generations and the calls around it still meet their peers."""
    xs, ws, dys = _inputs(rows, hl * tp, tp, dtype, 23)
    g = rtp.EmulatedTPGroup(tp, eps=1e-5, num_max_rows=512, timeout_s=5.0)
    try:
        y1 = g.forward(xs, ws)
        dxs, dws = g.backward(dys, xs, ws)
        y2 = g.forward(xs, ws)
        torch.cuda.synchronize()
        assert all(b.poll_error() == 0 for b in g.bufs)
        assert all(b.device_generation() == 4 for b in g.bufs)
        _check(dtype, xs, ws, dys, dxs, dws, 1e-5)
        name = NAMES[dtype]
        assert all(r["ok"] for r in check_against_oracle(name, xs, ws, 1e-5, y2, reference=False))
        for a, b in zip(y1, y2):
            assert torch.equal(a, b)
    finally:
        g.destroy()


@pytest.mark.parametrize("tp,rank", [(2, 0), (4, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_entry_point_backward_with_host_written_peer_slots(tp, rank, dtype):
    """rmsnorm_tp_backward on one GPU: the host writes the other ranks' sum(x^2)
    words (generation 0, buffer 0) and sum(dy * w * x) words (generation 1,
    buffer 1); this rank's two pushes must land in the stand-in peer mailboxes."""
    hl, rows, nmax = 1024, 200, 256
    name = NAMES[dtype]
    buf = rtp.TPCommBuffer(rank, tp, nmax)
    buf.allocate()
    buf.set_timeout(5.0)
    box_ptr, box_bytes = buf.mailbox()
    mine = device_view(box_ptr, box_bytes)
    fakes = {}
    for q in range(tp):
        if q != rank:
            fakes[q] = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
            buf.attach_peer(q, fakes[q].data_ptr())
    buf.finalize_setup()
    try:
        xs, ws, dys = _inputs(rows, hl * tp, tp, dtype, 33)
        X = [O.to_f32(name, to_np(t)).astype(np.float64) for t in xs]
        W = [O.to_f32(name, to_np(t)).astype(np.float64) for t in ws]
        DY = [O.to_f32(name, to_np(t)).astype(np.float64) for t in dys]
        s_part = [(x * x).sum(axis=-1).astype(np.float32) for x in X]
        d_part = [(dy * w * x).sum(axis=-1).astype(np.float32) for x, dy, w in zip(X, DY, W)]
        for q in range(tp):
            if q != rank:
                lo = slot_index(0, q, tp, nmax, 0)
                mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(s_part[q], rtp.tag_of(0))))
                lo = slot_index(1, q, tp, nmax, 0)
                mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(d_part[q], rtp.tag_of(1))))
        torch.cuda.synchronize()
        dx, dw = buf.launch_backward(dys[rank], xs[rank], ws[rank], hl * tp, 1e-6)
        torch.cuda.synchronize()
        assert buf.poll_error() == 0 and buf.device_generation() == 2
        want_dx, want_dw = O.backward_path([to_np(x) for x in xs], [to_np(d) for d in dys],
                                           [to_np(w) for w in ws], 1e-6, name)
        assert O.compare_backward(name, out_f32(name, dx), O.round_to(name, want_dx[rank]))["ok"]
        scale = O.dw_magnitude([to_np(x) for x in xs], [to_np(d) for d in dys], 1e-6, name)[rank]
        assert O.compare_backward(name, out_f32(name, dw), O.round_to(name, want_dw[rank]),
                                  scale)["ok"]
        for b, tag, part in ((0, rtp.tag_of(0), s_part), (1, rtp.tag_of(1), d_part)):
            lo = slot_index(b, rank, tp, nmax, 0)
            for f in fakes.values():
                words = f[lo:lo + rows].cpu().numpy().view(np.uint64)
                assert np.all((words >> np.uint64(32)) == tag)
                vals = (words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
                np.testing.assert_allclose(vals, part[rank], rtol=1e-5, atol=1e-4)
    finally:
        buf.destroy()


def test_autograd_at_tp1_uses_the_backward_kernel():
    m = rtp.FusedTPRMSNorm(2048, eps=1e-6)
    xs, ws, dys = _inputs(64, 2048, 1, torch.bfloat16, 43)
    x = xs[0].clone().requires_grad_()
    w = ws[0].clone().requires_grad_()
    y = m.forward_with_grad(x, w)
    (y.float() * dys[0].float()).sum().backward()
    dx, dw = rtp.local_rmsnorm_backward(dys[0], xs[0], ws[0], 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(x.grad, dx) and torch.equal(w.grad, dw)


def test_backward_missing_peer_times_out_then_reset_recovers():
    buf = rtp.TPCommBuffer(0, 2, 64)
    buf.allocate()
    buf.set_timeout(0.05)
    _, box_bytes = buf.mailbox()
    stand_in = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
    buf.attach_peer(1, stand_in.data_ptr())
    buf.finalize_setup()
    try:
        xs, ws, dys = _inputs(8, 2 * 256, 2, torch.bfloat16, 53)
        dx, dw = buf.launch_backward(dys[0], xs[0], ws[0], 512, 1e-6)
        torch.cuda.synchronize()                       # returns: the waits are bounded
        assert buf.poll_error() == _lib.STATUS_TIMEOUT
        assert buf.status()["src_rank"] == 1
        assert torch.isnan(dx.float()).all()
        with pytest.raises(rtp.RMSNormTPDeviceError):
            buf.launch_backward(dys[0], xs[0], ws[0], 512, 1e-6)
        buf.reset(0)
        assert buf.poll_error() == 0
    finally:
        buf.destroy()
