"""Generate the golden vectors of the TP RMSNorm from the REFERENCE itself.

Runs ``reference_tp_rmsnorm`` of haowen-han/RmsnormTP (bench_rmsnorm_tp.py:16-22,
its AllReduce path) on CPU tensors under gloo, one process per TP rank, and
stores every rank's inputs and outputs in ``golden.npz``. The reference checkout
only exists where the fixtures are made; the GPU box and the test suite read the
committed ``golden.npz`` only.

    python tests/golden/make_golden.py --reference <checkout of the reference>

Layout of golden.npz, per case ``<name>``:
    <name>/meta        json: dtype, tp, rows, local_hidden, eps, seed_base, stress
    <name>/x<r>, /w<r> rank r's inputs (f32 float32, bf16 uint16 bit patterns, f16 float16)
    <name>/y<r>        rank r's output of the reference (float32, as the reference returns it)
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from rmsnorm_tp_b200.workloads import NAME_DTYPES, make_slice  # noqa: E402

# name, dtype, tp, rows, local_hidden, eps, seed_base, stress
CASES = [
    ("f32_tp2_cfg1", "f32", 2, 16, 64, 1e-6, 0, False),
    ("f32_tp1", "f32", 1, 5, 80, 1e-6, 0, False),
    ("f32_tp2_ragged", "f32", 2, 7, 37, 1e-6, 0, False),
    ("f32_tp8", "f32", 8, 3, 32, 1e-6, 0, False),
    ("bf16_tp1", "bf16", 1, 6, 256, 1e-6, 1000, False),
    ("bf16_tp2", "bf16", 2, 8, 128, 1e-6, 1000, False),
    ("bf16_tp4", "bf16", 4, 8, 64, 1e-6, 1000, False),
    ("bf16_tp8_decode", "bf16", 8, 1, 128, 1e-5, 1000, False),
    ("bf16_tp4_stress", "bf16", 4, 32, 128, 1e-5, 1000, True),
    ("f16_tp2", "f16", 2, 8, 96, 1e-5, 1000, False),
    ("f16_tp4", "f16", 4, 4, 64, 1e-5, 1000, False),
    # outlier channels reach |x| > 256, where the reference squares overflow in fp16
    ("f16_tp2_overflow", "f16", 2, 16, 64, 1e-5, 1000, True),
]


def _load_reference(ref_root: str):
    path = os.path.join(ref_root, "bench_rmsnorm_tp.py")
    spec = importlib.util.spec_from_file_location("_ref_bench_rmsnorm_tp", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.reference_tp_rmsnorm


def _store(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def _rank_main(rank, tp, port, ref_root, case, outdir):
    name, dname, _, rows, hl, eps, seed_base, stress = case
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=tp)
    try:
        ref = _load_reference(ref_root)
        x, w = make_slice(rows, hl, NAME_DTYPES[dname], seed_base + rank, stress=stress,
                          stress_seed=seed_base)
        y = ref(x.clone(), w.clone(), eps, dist.group.WORLD)
        np.savez(os.path.join(outdir, f"{name}_{rank}.npz"), x=_store(x), w=_store(w),
                 y=y.to(torch.float32).numpy())
    finally:
        dist.destroy_process_group()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, help="checkout of haowen-han/RmsnormTP")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    ap.add_argument("--port", type=int, default=29611)
    args = ap.parse_args(argv)
    arrays = {}
    with tempfile.TemporaryDirectory() as tmp:
        for i, case in enumerate(CASES):
            name, dname, tp, rows, hl, eps, seed_base, stress = case
            mp.spawn(_rank_main, args=(tp, args.port + i, args.reference, case, tmp), nprocs=tp,
                     join=True)
            meta = dict(dtype=dname, tp=tp, rows=rows, local_hidden=hl, eps=eps,
                        seed_base=seed_base, stress=stress,
                        source="reference_tp_rmsnorm, bench_rmsnorm_tp.py:16-22, gloo CPU",
                        torch=torch.__version__)
            arrays[f"{name}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
            for r in range(tp):
                with np.load(os.path.join(tmp, f"{name}_{r}.npz")) as z:
                    for k in ("x", "w", "y"):
                        arrays[f"{name}/{k}{r}"] = z[k]
            print(f"{name}: tp={tp} rows={rows} hl={hl} {dname}", flush=True)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out} ({os.path.getsize(args.out)} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
