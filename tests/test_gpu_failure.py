"""Failure detection on the GPU without a GPU fault: a bounded wait runs out.

Rank 0 of a TP = 2 group whose peer mailbox is a device buffer that no rank
serves: the kernel pushes its partial there, waits for the peer's partial that
never comes, gives up after the timeout, records the failure and returns. The
context stays usable, later calls are refused until reset, and reset recovers.
"""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import check_against_oracle, device_view, pack_slots, slot_index, to_np
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200 import _lib
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


def _lonely_rank(timeout_s, nmax=64):
    buf = rtp.TPCommBuffer(0, 2, nmax)
    buf.allocate()
    buf.set_timeout(timeout_s)
    _, box_bytes = buf.mailbox()
    stand_in = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
    buf.attach_peer(1, stand_in.data_ptr())
    buf.finalize_setup()
    return buf, stand_in


@pytest.mark.parametrize("hl,dtype", [(512, torch.bfloat16), (37, torch.float32)])
def test_missing_peer_times_out_then_reset_recovers(family, hl, dtype):
    rows = 8
    buf, stand_in = _lonely_rank(0.05)
    try:
        xs, ws = make_group(rows, 2 * hl, 2, dtype, 11)
        x, w = xs[0].cuda(), ws[0].cuda()
        out = torch.zeros_like(x)
        buf.launch(out, x, w, 2 * hl, 1e-6)
        torch.cuda.synchronize()                       # returns: the wait is bounded
        assert buf.poll_error() == _lib.STATUS_TIMEOUT
        st = buf.status()
        assert st["code"] == _lib.STATUS_TIMEOUT
        assert st["src_rank"] == 1 and 0 <= st["row"] < rows
        assert st["expected_tag"] == rtp.tag_of(0) and st["seen_tag"] == 0
        assert st["generation"] == 0 and st["next_generation"] == 1
        assert torch.isnan(out.float()).all()          # failed rows are NaN, never stale
        with pytest.raises(rtp.RMSNormTPDeviceError):  # refused until reset
            buf.launch(out, x, w, 2 * hl, 1e-6)

        # the context is healthy: another kernel runs and is correct
        y = rtp.local_rmsnorm(x, w, 1e-6)
        torch.cuda.synchronize()
        dname = "bf16" if dtype == torch.bfloat16 else "f32"
        assert check_against_oracle(dname, [x], [w], 1e-6, [y])[0]["ok"]

        buf.reset(0)
        assert buf.poll_error() == 0 and buf.device_generation() == 0
        # now the peer's partials are there (written by the host, as its push would be)
        box_ptr, box_bytes = buf.mailbox()
        mine = device_view(box_ptr, box_bytes)
        p1 = O.partial_sums(to_np(xs[1]), dname)
        lo = slot_index(0, 1, 2, 64, 0)
        mine[lo:lo + rows].copy_(torch.from_numpy(pack_slots(p1, rtp.tag_of(0))))
        out2 = torch.empty_like(x)
        buf.launch(out2, x, w, 2 * hl, 1e-6)
        torch.cuda.synchronize()
        assert buf.poll_error() == 0
        want = O.fused_path([to_np(t) for t in xs], [to_np(t) for t in ws], 1e-6, dname)[0]
        res = O.compare(dname, O.to_f32(dname, to_np(out2)), O.round_to(dname, want))
        assert res["ok"], res
        # our partial reached the stand-in peer mailbox with the call's tag
        words = stand_in[slot_index(0, 0, 2, 64, 0):][:rows].cpu().numpy().view(np.uint64)
        assert np.all((words >> np.uint64(32)) == rtp.tag_of(0))
    finally:
        buf.destroy()


def test_ranks_that_disagree_on_the_generation_time_out_bounded(family):
    """Two emulated ranks whose generation counters differ (as after a rank
    skipped a call) push and await different tags; every wait ends at the
    timeout with an error status, inside the cooperative launch too."""
    g = rtp.EmulatedTPGroup(2, eps=1e-6, num_max_rows=64, timeout_s=0.05)
    try:
        g.bufs[1].reset(5)   # rank 1 thinks it is at call 5, rank 0 at call 0
        xs, ws = make_group(4, 2 * 256, 2, torch.bfloat16, 3, device="cuda")
        g.forward(xs, ws)
        torch.cuda.synchronize()
        codes = [b.poll_error() for b in g.bufs]
        assert _lib.STATUS_TIMEOUT in codes
        g.reset(0)
        outs = g.forward(xs, ws)
        torch.cuda.synchronize()
        assert [b.poll_error() for b in g.bufs] == [0, 0]
        assert all(r["ok"] for r in check_against_oracle("bf16", xs, ws, 1e-6, outs))
    finally:
        g.destroy()
