"""Multi-GPU worker for tests/test_gpu_multigpu.py (one process per GPU, NCCL
bootstrap, CUDA-IPC mailboxes over NVLink). Run under torchrun; rank 0 prints
"ALL OK" when every check passed on every rank.

Checks, on the real group (TP = world size):
1. the reference's own test cases (test_rmsnorm_tp.py:29-67 and :113-142):
   fp32, seed 42 + rank, weight ~ N(0,1), 128 rows at hidden 4096, then hidden
   {1024, 2048, 4096, 8192} x rows {1, 16, 128, 512} through ONE instance built
   with hidden_dim=4096 -- against the oracle of the AllReduce path;
2. bf16 / fp16 at the benchmark shapes, varying row counts from call to call,
   random 0-50 us host-side launch skew per rank;
3. CUDA-graph capture and replay of forward;
4. failure detection: rank 1 skips one call; rank 0's wait ends with a
   device-side timeout (bounded), forward is refused until the collective
   reset, and results are correct afterwards;
5. a prefill-size call (65536 rows, hidden 8192: the bulk-copy kernel), sampled
   rows gathered across ranks and checked by the oracle;
6. the fused residual add and the backward pass (two exchanges per row) between
   forward calls, checked by the oracle against every rank's inputs;
7. the one-hop round-trip probe between ranks 0 and 1;
8. every kernel family (batch, register, bulk) under both push encodings
   (packed {tag, partial} word; value + release-stored tag), decode to
   prefill row counts, including the fused residual add.
"""
import datetime
import os
import random
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from gpu_helpers import NAMES, to_np  # noqa: E402
from oracle import tp_rmsnorm as O  # noqa: E402
from rmsnorm_tp import FusedTPRMSNorm  # noqa: E402  (the drop-in import name)
import rmsnorm_tp_b200 as rtp  # noqa: E402
from rmsnorm_tp_b200.workloads import make_group  # noqa: E402

FAILS = []


def check(cond, msg):
    if not cond:
        FAILS.append(msg)
        print(f"[rank {dist.get_rank()}] FAIL {msg}", flush=True)


def compare_rank(dtype_name, xs, ws, eps, y, rank, what, reference=True):
    xn = [to_np(x) for x in xs]
    wn = [to_np(w) for w in ws]
    want = (O.allreduce_path if reference else O.fused_path)(xn, wn, eps, dtype_name)[rank]
    r = O.compare(dtype_name, O.to_f32(dtype_name, to_np(y)), O.round_to(dtype_name, want))
    check(r["ok"], f"{what}: {r}")
    return r


def reference_style_inputs(rows, hidden, tp, seed_offset=42):
    """Every rank's fp32 slice as the reference's test draws it (seed 42 + rank)."""
    xs, ws = [], []
    for r in range(tp):
        torch.manual_seed(seed_offset + r)
        xs.append(torch.randn(rows, hidden // tp, dtype=torch.float32))
        ws.append(torch.randn(hidden // tp, dtype=torch.float32))
    return xs, ws


def main():
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, tp = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    group = dist.group.WORLD
    dev = torch.device("cuda", local)

    # 1. the reference's test cases, one instance for every hidden size
    m = FusedTPRMSNorm(hidden_dim=4096, eps=1e-6, tp_group=group, num_max_rows=65536)
    m.comm_buf.set_timeout(10.0)
    xs, ws = reference_style_inputs(128, 4096, tp)
    y = m.forward(xs[rank].to(dev), ws[rank].to(dev))
    torch.cuda.synchronize()
    r = compare_rank("f32", xs, ws, 1e-6, y, rank, "test_correctness 128x4096 fp32")
    check(r["max_abs"] < 1e-3, "reference bound max-abs < 1e-3")
    for hidden in (1024, 2048, 4096, 8192):
        for rows in (1, 16, 128, 512):
            xs, ws = reference_style_inputs(rows, hidden, tp)
            y = m.forward(xs[rank].to(dev), ws[rank].to(dev))
            torch.cuda.synchronize()
            compare_rank("f32", xs, ws, 1e-6, y, rank, f"shapes hidden={hidden} rows={rows}")

    # 2. bf16 / fp16, varying rows, launch skew
    rng = random.Random(1234)   # same sequence of row counts on every rank
    skew = random.Random(rank)
    for call in range(60):
        dtype = (torch.bfloat16, torch.float16)[call % 2]
        rows = rng.choice([1, 2, 5, 64, 255, 256, 1000, 4096])
        xs, ws = make_group(rows, 4096, tp, dtype, 1000 + call)
        time.sleep(skew.random() * 50e-6)
        y = m.forward(xs[rank].to(dev), ws[rank].to(dev))
        if call % 10 == 9 or rows >= 1000:
            torch.cuda.synchronize()
            compare_rank(NAMES[dtype], xs, ws, 1e-6, y, rank, f"skewed call {call} rows={rows}")
    torch.cuda.synchronize()
    check(m.comm_buf.poll_error() == 0, "no device failure in the skewed calls")

    # 3. graph capture / replay
    xs, ws = make_group(256, 4096, tp, torch.bfloat16, 77)
    x, w = xs[rank].to(dev), ws[rank].to(dev)
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m.forward(x, w, out=out)
    s.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(3):
            m.forward(x, w, out=out)
    torch.cuda.synchronize()
    dist.barrier()
    for rep in range(4):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        compare_rank("bf16", xs, ws, 1e-6, out, rank, f"graph replay {rep}")
    del g
    check(m.comm_buf.poll_error() == 0, "no device failure in graph replays")

    # 4. failure detection: rank 1 skips one call
    m.comm_buf.set_timeout(0.3)
    torch.cuda.synchronize()
    dist.barrier()
    xs, ws = make_group(64, 4096, tp, torch.bfloat16, 5)
    x, w = xs[rank].to(dev), ws[rank].to(dev)
    if rank != 1:
        t0 = time.time()
        y = m.forward(x, w)
        torch.cuda.synchronize()
        check(time.time() - t0 < 10.0, "the wait is bounded")
        check(m.comm_buf.poll_error() == rtp._lib.STATUS_TIMEOUT, "timeout recorded")
        st = m.status()
        check(st["src_rank"] == 1, f"missing partial attributed to rank 1: {st}")
        check(bool(torch.isnan(y.float()).all()), "failed rows are NaN")
        try:
            m.forward(x, w)
            check(False, "forward must be refused after a device failure")
        except rtp.RMSNormTPDeviceError:
            pass
    m.reset()
    m.comm_buf.set_timeout(10.0)
    y = m.forward(x, w)
    torch.cuda.synchronize()
    compare_rank("bf16", xs, ws, 1e-6, y, rank, "after reset")
    check(m.comm_buf.poll_error() == 0, "clean after reset")

    # 5. prefill size (bulk-copy kernel over NVLink): 65536 rows of hidden 8192;
    # sampled rows of every rank's slice are gathered and checked by the oracle
    from rmsnorm_tp_b200.workloads import make_slice

    rows, hidden = 65536, 8192
    x, w = make_slice(rows, hidden // tp, torch.bfloat16, 2000 + rank, device=str(dev))
    y = m.forward(x, w)
    torch.cuda.synchronize()
    idx = torch.randperm(rows, generator=torch.Generator().manual_seed(7))[:64].to(dev)
    mine = [x.index_select(0, idx).contiguous(), w.contiguous()]
    xs_all = [torch.empty_like(mine[0]) for _ in range(tp)]
    ws_all = [torch.empty_like(mine[1]) for _ in range(tp)]
    dist.all_gather(xs_all, mine[0])
    dist.all_gather(ws_all, mine[1])
    compare_rank("bf16", [t.cpu() for t in xs_all], [t.cpu() for t in ws_all], 1e-6,
                 y.index_select(0, idx), rank, "prefill 65536 x 8192 (sampled rows)")
    del x, y

    # 6. fused residual add, backward, forward again (the generation advances 1 + 2 + 1)
    m.comm_buf.set_timeout(10.0)
    g0 = m.comm_buf.device_generation()
    for dtype in (torch.bfloat16, torch.float32):
        name = NAMES[dtype]
        rows, hidden = 300, 2048
        xs, ws = make_group(rows, hidden, tp, dtype, 3000)
        rs, _ = make_group(rows, hidden, tp, dtype, 3100)
        dys, _ = make_group(rows, hidden, tp, dtype, 3200)
        x, w, r, dy = (t[rank].to(dev) for t in (xs, ws, rs, dys))
        y = m.forward(x, w, residual=r)
        dx, dw = m.backward(dy, x, w)
        y2 = m.forward(x, w)
        torch.cuda.synchronize()
        ys, zs = O.allreduce_path_residual([to_np(t) for t in xs], [to_np(t) for t in rs],
                                           [to_np(t) for t in ws], 1e-6, name)
        check(np.array_equal(np.asarray(zs[rank]), to_np(r)), f"residual z {name}")
        res = O.compare(name, O.to_f32(name, to_np(y)), O.round_to(name, ys[rank]))
        check(res["ok"], f"residual forward {name}: {res}")
        want_dx, want_dw = O.backward_path([to_np(t) for t in xs], [to_np(t) for t in dys],
                                           [to_np(t) for t in ws], 1e-6, name)
        scale = O.dw_magnitude([to_np(t) for t in xs], [to_np(t) for t in dys], 1e-6, name)
        res = O.compare_backward(name, O.to_f32(name, to_np(dx)), O.round_to(name, want_dx[rank]))
        check(res["ok"], f"backward dx {name}: {res}")
        res = O.compare_backward(name, O.to_f32(name, to_np(dw)), O.round_to(name, want_dw[rank]),
                                 scale[rank])
        check(res["ok"], f"backward dw {name}: {res}")
        compare_rank(name, xs, ws, 1e-6, y2, rank, f"forward after backward {name}")
    check(m.comm_buf.poll_error() == 0, "no device failure in residual / backward calls")
    check(m.comm_buf.device_generation() == g0 + 8, "generation advanced by 4 per dtype")

    # 7. latency probe between ranks 0 and 1
    import ctypes
    from rmsnorm_tp_b200._lib import LIB

    res = torch.zeros(1, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    dist.barrier()
    if rank in (0, 1):
        rc = LIB.rmsnorm_tp_probe_roundtrip(m.comm_buf._comm, 1 - rank, 1000,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                            ctypes.c_void_p(res.data_ptr()))
        check(rc == 0, "probe launch")
    torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        ns = int(res.item())
        check(ns > 0, f"probe round trip {ns}")
        print(f"probe: store->poll round trip {ns} ns (one hop ~{ns / 2:.0f} ns)", flush=True)

    # 8. kernel families x push encodings over NVLink
    m.comm_buf.set_timeout(10.0)
    for family in ("batch", "register", "bulk"):
        for mode in ("packed", "release"):
            rtp.set_kernel_family(family)
            rtp.set_push_mode(mode)
            try:
                for rows in (1, 300, 4096):
                    xs, ws = make_group(rows, 4096, tp, torch.bfloat16, 5000 + rows)
                    rs, _ = make_group(rows, 4096, tp, torch.bfloat16, 5100 + rows)
                    x, w, r = (t[rank].to(dev) for t in (xs, ws, rs))
                    y = m.forward(x, w)
                    y2 = m.forward(x, w, residual=r)
                    torch.cuda.synchronize()
                    compare_rank("bf16", xs, ws, 1e-6, y, rank, f"{family}/{mode} rows={rows}")
                    want, zs = O.allreduce_path_residual(
                        [to_np(t) for t in xs], [to_np(t) for t in rs], [to_np(t) for t in ws],
                        1e-6, "bf16")
                    res = O.compare("bf16", O.to_f32("bf16", to_np(y2)),
                                    O.round_to("bf16", want[rank]))
                    check(res["ok"], f"{family}/{mode} residual rows={rows}: {res}")
            finally:
                rtp.set_kernel_family("auto")
                rtp.set_push_mode("packed")
    check(m.comm_buf.poll_error() == 0, "no device failure across families and encodings")

    m.destroy()
    fails = torch.tensor([len(FAILS)], device=dev)
    dist.all_reduce(fails)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("ALL OK" if int(fails.item()) == 0 else f"{int(fails.item())} FAILURES", flush=True)
    return 0 if int(fails.item()) == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
