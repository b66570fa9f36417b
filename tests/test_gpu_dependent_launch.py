"""Programmatic dependent launch: back-to-back forward kernels may be scheduled
while the previous one finishes, and must still see its writes (griddepcontrol.wait
before any global access). Each check runs a chain of calls whose input is the
previous call's output, or whose generation the previous call advanced, with no
synchronisation in between, and compares it with the same chain launched
without the dependency (bit-exact) and with the oracle."""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import device_view, out_f32, pack_slots, slot_index, to_np
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


@pytest.fixture
def dependent(request):
    before = rtp.get_dependent_launch()
    yield
    rtp.set_dependent_launch(before)


def _local_chain(x, w, n, graph):
    """y_1 = f(x), y_k = f(y_{k-1}), launched back to back on one stream."""
    outs = [torch.empty_like(x) for _ in range(n)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def run():
        src = x
        for o in outs:
            rtp.local_rmsnorm(src, w, 1e-6, o)
            src = o

    with torch.cuda.stream(s):
        run()
    s.synchronize()
    if graph:
        for o in outs:
            o.zero_()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            run()
        for o in outs:
            o.zero_()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        del g
    return [o.clone() for o in outs]


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("rows,hl", [(4096, 4096), (300, 1024), (16384, 4096)])
def test_chained_local_calls_see_the_previous_output(family, dependent, graph, rows, hl):
    xs, ws = make_group(rows, hl, 1, torch.bfloat16, 31, device="cuda")
    x, w = xs[0], ws[0]
    rtp.set_dependent_launch(True)
    on = _local_chain(x, w, 6, graph)
    rtp.set_dependent_launch(False)
    off = _local_chain(x, w, 6, graph)
    for a, b in zip(on, off):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    # first two links against the oracle (bf16 rounding of each link's input)
    src = to_np(x)
    wn = to_np(w)
    for k in range(2):
        want = O.fused_path([src], [wn], 1e-6, "bf16")[0]
        res = O.compare("bf16", out_f32("bf16", on[k]), O.round_to("bf16", want))
        assert res["ok"], (k, res)
        src = to_np(on[k])


def test_back_to_back_entry_point_calls_read_the_advanced_generation(family, dependent):
    """Call 1 must use buffer 1 / tag 1, which only the LAST CTA of call 0 makes
    current; the peers' partials of the two calls differ, so a call-1 kernel that
    read the generation early would take call 0's slots and produce other rows."""
    tp, rank, hl, rows, nmax = 2, 0, 4096, 512, 512
    rtp.set_dependent_launch(True)
    buf = rtp.TPCommBuffer(rank, tp, nmax)
    buf.allocate()
    buf.set_timeout(5.0)
    box_ptr, box_bytes = buf.mailbox()
    mine = device_view(box_ptr, box_bytes)
    stand_in = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
    buf.attach_peer(1, stand_in.data_ptr())
    buf.finalize_setup()
    try:
        calls = []
        for gen in range(2):
            xs, ws = make_group(rows, hl * tp, tp, torch.bfloat16, 50 + gen)
            p1 = O.partial_sums(to_np(xs[1]), "bf16")
            lo = slot_index(rtp.buffer_of(gen), 1, tp, nmax, 0)
            mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(p1, rtp.tag_of(gen))))
            want = O.fused_path([to_np(t) for t in xs], [to_np(t) for t in ws], 1e-6, "bf16")[0]
            calls.append((xs[0].cuda(), ws[0].cuda(), want))
        outs = [torch.empty_like(c[0]) for c in calls]
        torch.cuda.synchronize()
        for (x, w, _), o in zip(calls, outs):            # no synchronisation in between
            buf.launch(o, x, w, hl * tp, 1e-6)
        torch.cuda.synchronize()
        assert buf.poll_error() == 0
        assert buf.device_generation() == 2
        for k, ((_, _, want), o) in enumerate(zip(calls, outs)):
            res = O.compare("bf16", out_f32("bf16", o), O.round_to("bf16", want))
            assert res["ok"], (k, res)
    finally:
        buf.destroy()
