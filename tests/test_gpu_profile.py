"""In-kernel wait/timing counters (rmsnorm_tp_set_profile)."""
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import check_against_oracle
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu


def test_profile_counters_count_every_remote_wait(family):
    tp, rows, hl = 4, 300, 1024
    xs, ws = make_group(rows, hl * tp, tp, torch.bfloat16, 4, device="cuda")
    g = rtp.EmulatedTPGroup(tp, eps=1e-5, num_max_rows=rows, timeout_s=5.0)
    try:
        prof = rtp.profile_counters()
        g.bufs[0].set_profile(prof)          # the emulated launch uses rank 0's setting
        outs = g.forward(xs, ws)
        torch.cuda.synchronize()
        c = prof.cpu().tolist()
        # every rank waits once per (row, remote rank): fast + slow polls
        assert c[1] + c[2] == rows * tp * (tp - 1)
        assert c[0] >= 0 and (c[1] == 0 or c[0] > 0)
        assert 0 < c[3] <= c[4]
        # one launch: every CTA counted once, one span, no gap yet, scratch reset
        ctas = c[9]
        assert ctas > 0 and ctas % tp == 0
        assert c[11] == 1 and c[10] > 0 and c[13] == 0 and c[12] == 0
        # the launch's last CTA to arrive stamps its own end, at most the latest end
        assert c[14] == -1 and c[16] == 0 and c[3] < c[15] <= c[4]
        assert c[8] >= 0 and c[7] in (0, ctas)
        g.forward(xs, ws)
        torch.cuda.synchronize()
        c2 = prof.cpu().tolist()
        assert c2[9] == 2 * ctas and c2[11] == 2 and c2[13] == 1 and c2[12] >= 0
        assert c2[18] == ctas and c2[17] >= 0   # only the second launch's CTAs
        s = rtp.profile_summary(c2)
        assert s["launch_span_us"] > 0 and s["launch_gap_us"] is not None
        c = c2
        assert all(r["ok"] for r in check_against_oracle("bf16", xs, ws, 1e-5, outs))
        g.bufs[0].set_profile(None)
        g.forward(xs, ws)
        torch.cuda.synchronize()
        assert prof.cpu().tolist() == c      # switched off: untouched
    finally:
        g.destroy()
