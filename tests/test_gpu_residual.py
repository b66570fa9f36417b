"""GPU parity of the fused residual add + TP RMSNorm (through the C-ABI):
z = x + residual (rounded to x's dtype) written back into the residual, then the
norm of z. Checked against the oracle: the updated residual bit-exactly, the
output within the parity tolerance of the AllReduce path on z. TP = 1 (local
register / bulk / generic kernels), emulated TP = 2/4/8 (bulk / generic), the
real entry point with host-written peer slots, CUDA-graph replay, and a full-size
TP = 1 call."""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import NAMES, TORCH_DTYPES, device_view, out_f32, pack_slots, slot_index, to_np
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


def _inputs(rows, hidden, tp, dtype, seed):
    xs, ws = make_group(rows, hidden, tp, dtype, seed, device="cuda")
    rs, _ = make_group(rows, hidden, tp, dtype, seed + 77, device="cuda")
    return xs, ws, rs


def _check(dtype, xs, ws, rs_before, outs, rs_after, eps):
    name = NAMES[dtype]
    ys, zs = O.allreduce_path_residual([to_np(x) for x in xs], [to_np(r) for r in rs_before],
                                       [to_np(w) for w in ws], eps, name)
    for k, (y, z, o, r) in enumerate(zip(ys, zs, outs, rs_after)):
        assert np.array_equal(np.asarray(z), to_np(r)), f"rank {k}: updated residual differs"
        res = O.compare(name, out_f32(name, o), O.round_to(name, y))
        assert res["ok"], f"rank {k}: {res}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hidden", [37, 96, 512, 4096, 8192])
@pytest.mark.parametrize("rows", [1, 7, 300, 2500])
def test_local_residual(family, dtype, hidden, rows):
    xs, ws, rs = _inputs(rows, hidden, 1, dtype, 11)
    before = rs[0].clone()
    y = rtp.local_rmsnorm(xs[0], ws[0], 1e-6, residual=rs[0])
    torch.cuda.synchronize()
    _check(dtype, xs, ws, [before], [y], rs, 1e-6)


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hl,rows", [(64, 5), (512, 300), (1024, 1), (2048, 129), (4096, 64),
                                     (8192, 9), (37, 40)])
def test_emulated_group_residual(tp, dtype, hl, rows):
    xs, ws, rs = _inputs(rows, hl * tp, tp, dtype, 21)
    before = [r.clone() for r in rs]
    g = rtp.EmulatedTPGroup(tp, eps=1e-5, num_max_rows=512, timeout_s=5.0)
    try:
        outs = g.forward(xs, ws, residuals=rs)
        outs2 = g.forward(xs, ws, residuals=[b.clone() for b in before])   # second generation
        torch.cuda.synchronize()
        assert all(b.poll_error() == 0 for b in g.bufs)
        _check(dtype, xs, ws, before, outs, rs, 1e-5)
        for a, b in zip(outs, outs2):
            assert torch.equal(a, b)
    finally:
        g.destroy()


def test_module_residual_at_tp1_and_overlap_rejected():
    m = rtp.FusedTPRMSNorm(4096, eps=1e-6)
    xs, ws, rs = _inputs(64, 4096, 1, torch.bfloat16, 5)
    before = rs[0].clone()
    y = m.forward(xs[0], ws[0], residual=rs[0])
    torch.cuda.synchronize()
    _check(torch.bfloat16, xs, ws, [before], [y], rs, 1e-6)
    with pytest.raises(rtp.RMSNormTPError):
        m.forward(xs[0], ws[0], out=rs[0], residual=rs[0])


@pytest.mark.parametrize("tp,rank", [(2, 1), (4, 0), (8, 3)])
@pytest.mark.parametrize("hl,rows", [(2048, 100), (4096, 3)])
def test_entry_point_residual_with_host_written_peer_slots_and_graph(tp, rank, hl, rows):
    """rmsnorm_tp_forward_residual on one GPU with stand-in peers: the pushed
    partials are those of z, eager and replayed from a CUDA graph (two
    generations back to back)."""
    nmax = 512
    dtype = torch.bfloat16
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
        xs, ws, rs = _inputs(rows, hl * tp, tp, dtype, 31)
        before = [r.clone() for r in rs]
        zs = [O.residual_add(to_np(x), to_np(r), "bf16") for x, r in zip(xs, before)]
        partials = [O.partial_sums(z, "bf16") for z in zs]

        def write_peer_slots(gen):
            for q in range(tp):
                if q != rank:
                    lo = slot_index(rtp.buffer_of(gen), q, tp, nmax, 0)
                    mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(partials[q], rtp.tag_of(gen))))

        x, w = xs[rank], ws[rank]
        res = rs[rank]
        out = torch.empty_like(x)
        write_peer_slots(0)
        write_peer_slots(1)
        torch.cuda.synchronize()
        buf.launch(out, x, w, hl * tp, 1e-6, residual=res)
        torch.cuda.synchronize()
        assert buf.poll_error() == 0
        assert np.array_equal(to_np(res), np.asarray(zs[rank]))
        want = O.fused_path([z for z in zs], [to_np(t) for t in ws], 1e-6, "bf16")[rank]
        assert O.compare("bf16", out_f32("bf16", out), O.round_to("bf16", want))["ok"]
        words = fakes[(rank + 1) % tp][slot_index(0, rank, tp, nmax, 0):][:rows].cpu().numpy()
        vals = (words.view(np.uint64) & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
        np.testing.assert_allclose(vals, partials[rank], rtol=2e-6)
        # generation 1 from a CUDA graph, residual restored first
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        res.copy_(before[rank])
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            buf.launch(out, x, w, hl * tp, 1e-6, residual=res)
        res.copy_(before[rank])
        out.zero_()
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert buf.poll_error() == 0 and buf.device_generation() == 2
        assert np.array_equal(to_np(res), np.asarray(zs[rank]))
        assert O.compare("bf16", out_f32("bf16", out), O.round_to("bf16", want))["ok"]
        del graph
    finally:
        buf.destroy()


def test_local_residual_full_size_bulk():
    """65536 x 4096 bf16 at TP = 1 (512 MiB of x: the bulk kernel with x and
    residual tiles): the whole updated residual against torch's x + r on the GPU,
    sampled rows of the output against the oracle."""
    rows, hidden = 65536, 4096
    xs, ws, rs = _inputs(rows, hidden, 1, torch.bfloat16, 41)
    assert rtp.plan(rows, hidden, torch.bfloat16)["variant"] >= 100
    want_z = xs[0] + rs[0]
    idx = torch.from_numpy(np.sort(np.random.default_rng(3).choice(rows, 96, replace=False))).cuda()
    before = rs[0].index_select(0, idx)
    y = rtp.local_rmsnorm(xs[0], ws[0], 1e-6, residual=rs[0])
    torch.cuda.synchronize()
    assert torch.equal(rs[0], want_z)
    _check(torch.bfloat16, [xs[0].index_select(0, idx)], ws, [before], [y.index_select(0, idx)],
           [rs[0].index_select(0, idx)], 1e-6)
