"""GPU parity of the fused row-parallel linear -> reduce-scatter -> (residual
add) -> TP RMSNorm kernel (tcgen05 GEMM tiles stored into the owner's receive
buffer, then the norm with the one-scalar-per-row exchange), through the C ABI,
against the oracle of the unfused pipeline (oracle/tp_rmsnorm.py
linear_rs_norm_path: fp32 GEMM, partial rounded to the dtype, rank-order sum,
the reference's AllReduce norm). TP > 1 runs every rank in one cooperative
launch on one GPU (EmulatedTPLinearGroup); TP = 1 runs the module.

Tolerance: the parity bar of the suite (bf16/fp16: atol 1e-2 + rtol 1.6e-2);
the kernel's GEMM accumulates in another order than the oracle's, which can
move a partial by one unit of the dtype before the sum.
"""
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import NAMES, to_np
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200.workloads import make_group, make_linear_group

pytestmark = pytest.mark.gpu


def _check(name, as_, lws, gs, eps, outs, rs=None, rs_after=None):
    want, zs = O.linear_rs_norm_path([to_np(a) for a in as_], [to_np(w) for w in lws],
                                     [to_np(g) for g in gs], eps, name,
                                     None if rs is None else [to_np(r) for r in rs])
    for r, (o, w) in enumerate(zip(outs, want)):
        res = O.compare(name, O.to_f32(name, to_np(o)), O.round_to(name, w))
        assert res["ok"], (r, res)
    if rs_after is not None:   # the updated residual z = x + residual, within one unit of x
        for r, (z, zw) in enumerate(zip(rs_after, zs)):
            res = O.compare(name, O.to_f32(name, to_np(z)), O.to_f32(name, zw))
            assert res["ok"], ("residual", r, res)


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k,hl", [(1, 64, 128), (100, 128, 128), (128, 256, 256),
                                       (300, 512, 256)])
def test_emulated_group_matches_oracle(tp, dtype, rows, k, hl):
    name = NAMES[dtype]
    hidden = hl * tp
    as_, lws, gs = make_linear_group(rows, k, hidden, tp, dtype, 7 * rows + k, device="cuda")
    g = rtp.EmulatedTPLinearGroup(tp, hidden, eps=1e-5, num_max_rows=512, timeout_s=5.0)
    try:
        for _ in range(3):   # both generation buffers, and a buffer reused
            outs = g.forward(as_, lws, gs)
        torch.cuda.synchronize()
        assert all(b.poll_error() == 0 for b in g.bufs)
    finally:
        g.destroy()
    _check(name, as_, lws, gs, 1e-5, outs)


@pytest.mark.parametrize("tp", [2, 8])
@pytest.mark.parametrize("rows", [7, 256])
def test_emulated_group_residual(tp, rows):
    name, dtype, k, hidden = "bf16", torch.bfloat16, 256, 256 * tp
    as_, lws, gs = make_linear_group(rows, k, hidden, tp, dtype, 99 + rows, device="cuda")
    rs, _ = make_group(rows, hidden, tp, dtype, 5 + rows, device="cuda")
    rs_before = [r.clone() for r in rs]
    g = rtp.EmulatedTPLinearGroup(tp, hidden, eps=1e-6, num_max_rows=rows, timeout_s=5.0)
    try:
        outs = g.forward(as_, lws, gs, residuals=rs)
        torch.cuda.synchronize()
        assert all(b.poll_error() == 0 for b in g.bufs)
    finally:
        g.destroy()
    _check(name, as_, lws, gs, 1e-6, outs, rs_before, rs)


def test_rows_vary_between_calls_and_tiles_of_every_owner():
    """Row counts that change from call to call (partial last row block) on one
    group; hidden of several 128-column tiles per owner."""
    tp, k, hidden, dtype = 4, 128, 4 * 384, torch.bfloat16
    g = rtp.EmulatedTPLinearGroup(tp, hidden, eps=1e-5, num_max_rows=600, timeout_s=5.0)
    try:
        for call, rows in enumerate((600, 1, 129, 257, 128)):
            as_, lws, gs = make_linear_group(rows, k, hidden, tp, dtype, 1000 + call, device="cuda")
            outs = g.forward(as_, lws, gs)
            torch.cuda.synchronize()
            _check("bf16", as_, lws, gs, 1e-5, outs)
        assert all(b.device_generation() == 5 for b in g.bufs)
    finally:
        g.destroy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k,hidden", [(200, 512, 1024),    # 64-column tiles (few row blocks)
                                           (1280, 128, 2048),   # 128-column tiles
                                           (2048, 256, 4096)])  # 256-column tiles
def test_tp1_module(dtype, rows, k, hidden):
    """TP = 1: the GEMM and the norm without an exchange, at every tile width
    (the widest that still gives each of the 148 SMs a tile)."""
    name = NAMES[dtype]
    as_, lws, gs = make_linear_group(rows, k, hidden, 1, dtype, 3, device="cuda")
    m = rtp.FusedTPLinearRMSNorm(hidden, eps=1e-5, num_max_rows=rows)
    try:
        y = m.forward(as_[0], lws[0], gs[0])
        torch.cuda.synchronize()
    finally:
        m.destroy()
    _check(name, as_, lws, gs, 1e-5, [y])


def test_graph_capture_of_the_module():
    rows, k, hidden, dtype = 64, 256, 512, torch.bfloat16
    as_, lws, gs = make_linear_group(rows, k, hidden, 1, dtype, 11, device="cuda")
    m = rtp.FusedTPLinearRMSNorm(hidden, eps=1e-5, num_max_rows=rows)
    out = torch.empty(rows, hidden, dtype=dtype, device="cuda")
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            m.forward(as_[0], lws[0], gs[0], out=out)
        s.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            m.forward(as_[0], lws[0], gs[0], out=out)
        for _ in range(3):
            out.zero_()
            gr.replay()
            torch.cuda.synchronize()
            _check("bf16", as_, lws, gs, 1e-5, [out])
        del gr
    finally:
        m.destroy()


def test_output_overlapping_an_input_is_rejected_and_generation_unchanged():
    """out (or the residual) is written while other CTAs may still read a and the
    weights: an overlap is an argument error, raised before any launch, and a
    rejected call advances neither the host's nor the device's generation."""
    rows, k, hidden, dtype = 64, 128, 256, torch.bfloat16
    as_, lws, gs = make_linear_group(rows, k, hidden, 1, dtype, 5, device="cuda")
    m = rtp.FusedTPLinearRMSNorm(hidden, eps=1e-5, num_max_rows=rows)
    try:
        big = torch.empty(rows * max(k, hidden) * 2, dtype=dtype, device="cuda")
        a = big[: rows * k].view(rows, k)
        a.copy_(as_[0])
        with pytest.raises(rtp.RMSNormTPError, match="overlaps"):
            m.forward(a, lws[0], gs[0], out=big[: rows * hidden].view(rows, hidden))
        with pytest.raises(rtp.RMSNormTPError, match="overlaps"):
            m.forward(a, lws[0], gs[0], residual=big[64: 64 + rows * hidden].view(rows, hidden))
        torch.cuda.synchronize()
        assert m.comm_buf.generation == 0 and m.comm_buf.device_generation() == 0
        y = m.forward(a, lws[0], gs[0])        # disjoint output: runs
        torch.cuda.synchronize()
        # TP = 1 makes no exchange, so only the host's count moves
        assert m.comm_buf.generation == 1 and m.comm_buf.device_generation() == 0
    finally:
        m.destroy()
    _check("bf16", as_, lws, gs, 1e-5, [y])
