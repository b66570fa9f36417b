"""rmsnorm_tp_forward_group_static: the TP group on one GPU with no device
allocation (static scratch), for callers that may not call cudaMalloc --
serving runtimes with a memory pool fixed at start-up, plugin hosts that pass a
kernel only its inputs and outputs.

Called through the C ABI and checked against the existing entry point
(rmsnorm_tp_forward_emulated, which allocates its mailboxes) on the same
inputs, on two calls in a row, within the parity tolerance of the suite. This
file is collected last so a failure here stops a `-x` run only after every
other test has run; it passes alone in a fresh process too.
"""
import ctypes

import pytest
import torch

import rmsnorm_tp_b200 as rtp
from gpu_helpers import NAMES, check_against_oracle, out_f32
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200 import _lib
from rmsnorm_tp_b200.workloads import make_group

pytestmark = pytest.mark.gpu

SCRATCH = 4 << 20   # RMSNORM_TP_STATIC_SCRATCH_BYTES


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _call_static(xs, ws, outs, eps):
    tp = len(xs)
    rows, hl = xs[0].shape
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.LIB.rmsnorm_tp_forward_group_static(
        tp, _ptrs(outs), _ptrs(xs), _ptrs(ws), rows, hl, rtp.dtype_code(xs[0].dtype),
        float(eps), ctypes.c_void_p(stream))


@pytest.mark.parametrize("tp,rows,hl,dtype", [
    (2, 300, 1024, torch.bfloat16),
    (4, 257, 512, torch.float32),
    (8, 64, 1024, torch.float16),
    (3, 100, 37, torch.bfloat16),      # width not a multiple of 16 bytes: generic kernel
])
def test_static_scratch_entry_point_matches_allocating_one(tp, rows, hl, dtype):
    eps = 1e-5
    g = rtp.EmulatedTPGroup(tp, eps=eps, num_max_rows=rows, timeout_s=5.0)
    try:
        for call in range(2):                      # two calls in a row
            xs, ws = make_group(rows, hl * tp, tp, dtype, 500 + 17 * call + tp, device="cuda")
            want = g.forward(xs, ws)
            outs = [torch.full_like(x, float("nan")) for x in xs]
            rc = _call_static(xs, ws, outs, eps)
            assert rc == 0, _lib.last_error()
            torch.cuda.synchronize()
            name = NAMES[dtype]
            for r in range(tp):
                res = O.compare(name, out_f32(name, outs[r]), out_f32(name, want[r]))
                assert res["ok"], (call, r, res)
            assert all(res["ok"] for res in check_against_oracle(name, xs, ws, eps, outs))
    finally:
        g.destroy()


def test_static_scratch_rejects_sizes_beyond_its_limit():
    tp, hl = 8, 64
    rows_ok = (SCRATCH - 256 * tp) // (16 * tp * tp)
    xs, ws = make_group(rows_ok + 1, hl * tp, tp, torch.bfloat16, 3, device="cuda")
    outs = [torch.empty_like(x) for x in xs]
    rc = _call_static(xs, ws, outs, 1e-6)
    assert rc == _lib.ERR_ROWS
    assert "static scratch holds" in _lib.last_error()
    # the largest size that fits is accepted and correct
    xs = [x[:rows_ok].contiguous() for x in xs]
    outs = [torch.empty_like(x) for x in xs]
    assert _call_static(xs, ws, outs, 1e-6) == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert all(res["ok"] for res in check_against_oracle("bf16", xs, ws, 1e-6, outs))
