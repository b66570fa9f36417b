"""CUDA-graph capture of the forward call. The generation lives on the device
and the kernel advances it, so a replayed launch uses the next buffer and tag
(the reference passes the generation as a kernel argument, which a captured
graph would freeze: rmsnorm_tp/__init__.py:113, csrc/rmsnorm_tp.cu:61)."""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import check_against_oracle, device_view, out_f32, pack_slots, slot_index, to_np
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


def test_graph_replays_advance_the_generation_on_the_entry_point(family):
    tp, rank, hl, rows, nmax = 4, 1, 1024, 16, 64
    buf = rtp.TPCommBuffer(rank, tp, nmax)
    buf.allocate()
    buf.set_timeout(5.0)
    box_ptr, box_bytes = buf.mailbox()
    mine = device_view(box_ptr, box_bytes)
    fakes = []
    for q in range(tp):
        if q != rank:
            f = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
            fakes.append(f)
            buf.attach_peer(q, f.data_ptr())
    buf.finalize_setup()
    try:
        xs, ws = make_group(rows, hl * tp, tp, torch.bfloat16, 21)
        x, w = xs[rank].cuda(), ws[rank].cuda()
        out = torch.empty_like(x)
        partials = [O.partial_sums(to_np(t), "bf16") for t in xs]
        want = O.fused_path([to_np(t) for t in xs], [to_np(t) for t in ws], 1e-5, "bf16")[rank]

        def write_peer_slots(gen):
            for q in range(tp):
                if q != rank:
                    lo = slot_index(rtp.buffer_of(gen), q, tp, nmax, 0)
                    mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(partials[q], rtp.tag_of(gen))))

        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            write_peer_slots(0)
            buf.launch(out, x, w, hl * tp, 1e-5)       # warm-up (generation 0)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            buf.launch(out, x, w, hl * tp, 1e-5)
        for gen in range(1, 6):                         # replays use generations 1..5
            out.zero_()
            write_peer_slots(gen)
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            assert buf.poll_error() == 0, gen
            res = O.compare("bf16", out_f32("bf16", out), O.round_to("bf16", want))
            assert res["ok"], (gen, res)
        assert buf.device_generation() == 6
        del graph
    finally:
        buf.destroy()


def test_graph_of_local_kernel(family):
    xs, ws = make_group(300, 4096, 1, torch.bfloat16, 9, device="cuda")
    x, w = xs[0], ws[0]
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        rtp.local_rmsnorm(x, w, 1e-6, out)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        rtp.local_rmsnorm(x, w, 1e-6, out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert check_against_oracle("bf16", [x], [w], 1e-6, [out])[0]["ok"]
