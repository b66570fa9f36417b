"""The reference's push encoding (value, then a release-stored tag; read with an
acquire of the tag -- csrc/rmsnorm_tp.cu:102-115, :121-138), kept beside the
packed 64-bit {tag, partial} word for measured comparison: both encodings give
the oracle's results with every kernel family that exchanges partials."""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import (TORCH_DTYPES, check_against_oracle, device_view, out_f32, pack_slots,
                         slot_index, to_np)
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["packed", "release"])
def push_mode(request):
    rtp.set_push_mode(request.param)
    yield request.param
    rtp.set_push_mode("packed")


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("hl,rows", [(512, 1), (1024, 300), (2048, 4096)])
def test_emulated_group_both_encodings(family, push_mode, tp, dtype, hl, rows):
    xs, ws = make_group(rows, hl * tp, tp, TORCH_DTYPES[dtype], 11 * hl + rows, device="cuda")
    g = rtp.EmulatedTPGroup(tp, eps=1e-5, num_max_rows=rows, timeout_s=5.0)
    try:
        for _ in range(3):   # both buffers, and a buffer reused
            outs = g.forward(xs, ws)
        torch.cuda.synchronize()
        assert all(b.poll_error() == 0 for b in g.bufs)
    finally:
        g.destroy()
    res = check_against_oracle(dtype, xs, ws, 1e-5, outs)
    assert all(r["ok"] for r in res), res


@pytest.mark.parametrize("hl,rows", [(1024, 1), (512, 77), (2048, 300)])
def test_entry_point_release_encoding_writes_value_then_tag(family, hl, rows):
    """rmsnorm_tp_forward at TP = 4 on one GPU with host-written peer words: in
    the release encoding the slot has the same layout ({tag} in the high half,
    the partial in the low half), so the peers' words written by the host are
    read correctly and this rank's pushes arrive whole."""
    tp, rank, nmax, dtype = 4, 2, 512, "bf16"
    rtp.set_push_mode("release")
    buf = rtp.TPCommBuffer(rank, tp, nmax)
    buf.allocate()
    buf.set_timeout(5.0)
    try:
        box_ptr, box_bytes = buf.mailbox()
        mine = device_view(box_ptr, box_bytes)
        fakes = {}
        for q in range(tp):
            if q != rank:
                fakes[q] = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
                buf.attach_peer(q, fakes[q].data_ptr())
        buf.finalize_setup()
        for call in range(3):
            xs, ws = make_group(rows, hl * tp, tp, TORCH_DTYPES[dtype], 31 * call + rows)
            tag, b = rtp.tag_of(call), rtp.buffer_of(call)
            partials = [O.partial_sums(to_np(x), dtype) for x in xs]
            for q in range(tp):
                if q != rank:
                    lo = slot_index(b, q, tp, nmax, 0)
                    mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(partials[q], tag)))
            x, w = xs[rank].cuda(), ws[rank].cuda()
            out = torch.empty_like(x)
            buf.launch(out, x, w, hl * tp, 1e-5)
            torch.cuda.synchronize()
            assert buf.poll_error() == 0
            want = O.fused_path([to_np(t) for t in xs], [to_np(t) for t in ws], 1e-5, dtype)[rank]
            res = O.compare(dtype, out_f32(dtype, out), O.round_to(dtype, want))
            assert res["ok"], (call, res)
            lo = slot_index(b, rank, tp, nmax, 0)
            for q, f in fakes.items():
                words = f[lo:lo + rows].cpu().numpy().view(np.uint64)
                assert np.all((words >> np.uint64(32)) == tag)
                vals = (words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
                np.testing.assert_allclose(vals, partials[rank], rtol=2e-6)
    finally:
        rtp.set_push_mode("packed")
        buf.destroy()
