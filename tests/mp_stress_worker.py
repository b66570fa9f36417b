"""Stress run of the fused TP RMSNorm on a real multi-GPU group (one process per
GPU, NCCL bootstrap, CUDA-IPC mailboxes over NVLink). Run under torchrun:

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        tests/mp_stress_worker.py --calls 100000

The configuration is the stress row of the benchmark configurations: hidden
16384 split over the ranks (2048 per rank at TP 8), bf16, 65536 rows
(= num_max_rows), x ~ N(0,1) with 1 % of the channels scaled by 100 and 1 % of
the rows all zero, weight ~ 1 + 0.1 N(0,1), eps 1e-5. The generation starts
just below the 32-bit tag wrap (reset to 2^32 - 50 on every rank), so the tag
wraps early in the run -- the hazard of the reference's `<` poll
(csrc/rmsnorm_tp.cu:128), which also accepts a newer generation for the
current one. Before every call each rank puts a spin kernel of a random
0-50 us into its stream (torch.cuda._sleep), so the ranks reach each call with
random skew on the device timeline. Every 10^4 calls, sampled rows of every
rank are gathered to rank 0 and checked by the oracle of the reference's
AllReduce path. At the end every rank reports its device failure record (must
be empty) and its generation counter (must equal 2^32 - 50 + calls).

Rank 0 prints one JSON line starting with "STRESS " and "STRESS OK" if every
check passed on every rank.
"""
import argparse
import datetime
import json
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from gpu_helpers import to_np  # noqa: E402
from oracle import tp_rmsnorm as O  # noqa: E402
from rmsnorm_tp import FusedTPRMSNorm  # noqa: E402  (the drop-in import name)
import rmsnorm_tp_b200 as rtp  # noqa: E402
from rmsnorm_tp_b200.workloads import BY_NAME, make_slice  # noqa: E402

START_GENERATION = 2**32 - 50


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--calls", type=int, default=100000)
    ap.add_argument("--check-every", type=int, default=10000)
    ap.add_argument("--max-skew-us", type=float, default=50.0)
    ap.add_argument("--rows", type=int, default=None, help="fewer rows (shorter runs)")
    args = ap.parse_args()

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
    rank, tp = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = BY_NAME["stress"]
    rows = args.rows or cfg.rows[0]
    hl = cfg.hidden // tp
    x, w = make_slice(rows, hl, cfg.dtype, cfg.seed_base + rank, stress=True,
                      stress_seed=cfg.seed_base, device=str(dev))
    out = torch.empty_like(x)
    zero_rows = (x == 0).all(dim=1)
    zr = zero_rows.to(torch.int32)
    dist.all_reduce(zr, op=dist.ReduceOp.MIN)          # rows zero across the whole hidden dim
    zero_all = zr.bool()

    m = FusedTPRMSNorm(cfg.hidden, eps=cfg.eps, tp_group=dist.group.WORLD, num_max_rows=rows,
                       timeout_s=10.0)
    m.reset(START_GENERATION)
    mhz = 1965.0   # spin-kernel cycles per microsecond at the B200's maximum SM clock
    rng = np.random.default_rng(1234 + rank)
    idx = torch.from_numpy(np.sort(np.random.default_rng(7).choice(rows, 64, replace=False))).to(dev)
    checks, fails = [], []

    def check_now(call):
        torch.cuda.synchronize()
        xs = [torch.empty(64, hl, dtype=x.dtype, device=dev) for _ in range(tp)]
        ys = [torch.empty_like(xs[0]) for _ in range(tp)]
        ws = [torch.empty_like(w) for _ in range(tp)]
        dist.all_gather(xs, x.index_select(0, idx).contiguous())
        dist.all_gather(ys, out.index_select(0, idx).contiguous())
        dist.all_gather(ws, w)
        finite = bool(torch.isfinite(out.float()).all())
        zeros_ok = bool((out[zero_all] == 0).all())
        ok = finite and zeros_ok
        rec = {"call": call, "finite": finite, "zero_rows_zero": zeros_ok}
        if rank == 0:
            want = O.allreduce_path([to_np(t) for t in xs], [to_np(t) for t in ws], cfg.eps, "bf16")
            res = [O.compare("bf16", O.to_f32("bf16", to_np(ys[r])), O.round_to("bf16", want[r]))
                   for r in range(tp)]
            rec["oracle_ok"] = all(r["ok"] for r in res)
            rec["max_abs"] = max(r["max_abs"] for r in res)
            ok = ok and rec["oracle_ok"]
        checks.append(rec)
        if not ok:
            fails.append(rec)

    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    skews = rng.random(args.calls) * args.max_skew_us
    for call in range(args.calls):
        cycles = int(skews[call] * mhz)
        if cycles > 0:
            torch.cuda._sleep(cycles)
        m.forward(x, w, out=out)
        if (call + 1) % args.check_every == 0 or call + 1 == args.calls:
            check_now(call + 1)
        elif call % 256 == 255:
            torch.cuda.synchronize()      # keep the host within a bounded distance of the GPU
    e1.record()
    torch.cuda.synchronize()
    gpu_ms = e0.elapsed_time(e1)
    wall = time.perf_counter() - t0
    st = m.status()
    gen = m.comm_buf.device_generation()
    mine = {"rank": rank, "device_status": int(st["code"]), "generation": int(gen),
            "expected_generation": START_GENERATION + args.calls,
            "poll_error": int(m.comm_buf.poll_error())}
    everyone = [None] * tp
    dist.all_gather_object(everyone, mine)
    nf = torch.tensor([len(fails)], device=dev)
    dist.all_reduce(nf)
    m.destroy()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        ok = int(nf.item()) == 0 and all(
            e["device_status"] == 0 and e["poll_error"] == 0 and
            e["generation"] == e["expected_generation"] for e in everyone)
        summary = {
            "config": {"hidden": cfg.hidden, "tp": tp, "local_hidden": hl, "rows": rows,
                       "dtype": "bf16", "eps": cfg.eps, "stress_pattern": "1% channels x100, "
                       "1% rows zero", "kernel_family": rtp.get_kernel_family()},
            "calls": args.calls, "start_generation": START_GENERATION,
            "tag_wrap_at_call": (2**32 - 1) - START_GENERATION,
            "skew": f"spin kernel of U(0, {args.max_skew_us}) us before every call, per rank",
            "gpu_ms": round(gpu_ms, 1), "wall_s": round(wall, 2),
            "us_per_call_incl_skew": round(gpu_ms * 1e3 / args.calls, 2),
            "ranks": everyone, "checks": checks, "failed_checks": int(nf.item()), "ok": ok}
        print("STRESS " + json.dumps(summary), flush=True)
        print("STRESS OK" if ok else "STRESS FAILED", flush=True)
        return 0 if ok else 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
