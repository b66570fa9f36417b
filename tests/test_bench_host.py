"""Host logic of bench.py, on the CPU.

* the reference arm never maps this repository's CUDA library into its process
  and prints the same `config` as our arm;
* the parity check that bench.py runs after its timed region passes for a
  module that computes the reference's AllReduce path, and fails when some rows of
  one rank are wrong (a planted mistake), on one rank and on two gloo ranks.
"""
import json
import os
import subprocess
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_reference_arm_does_not_load_the_cuda_library():
    code = (
        "import atexit, runpy, sys\n"
        "def chk():\n"
        "    maps = open('/proc/self/maps').read()\n"
        "    print('LIBRARY_MAPPED' if 'librmsnorm_tp_b200' in maps else 'LIBRARY_NOT_MAPPED')\n"
        "    print('PACKAGE_IMPORTED' if 'rmsnorm_tp_b200' in sys.modules else 'PACKAGE_NOT_IMPORTED')\n"
        "atexit.register(chk)\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1',\n"
        "            '--rows', '64', '--hidden', '256']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n")
    res = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    assert "LIBRARY_NOT_MAPPED" in res.stdout and "PACKAGE_NOT_IMPORTED" in res.stdout
    line = json.loads(res.stdout.splitlines()[0])
    assert line["impl"] == "reference"
    args = bench.parse_args(["--rows", "64", "--hidden", "256"])
    assert line["config"] == bench.bench_config(bench.workload_of(args), 1)


class _OracleModule:
    """Stands in for FusedTPRMSNorm on CPU tensors: the reference's AllReduce path
    (oracle/torch_port.py) with an optional planted mistake in some rows of one rank."""

    def __init__(self, eps, rank, bad_rank=None, bad_what=None):
        self.eps, self.rank = eps, rank
        self.bad_rank, self.bad_what = bad_rank, bad_what

    def _plant(self, t, what):
        if self.rank == self.bad_rank and self.bad_what == what:
            t = t.clone()
            t[::7] = t[::7] * 1.5 + 0.25     # every 7th row: some are among the sampled rows
        return t

    def forward(self, x, w, out=None, residual=None):
        from oracle import torch_port

        if residual is not None:
            residual.copy_((x.float() + residual.float()).to(x.dtype))
            x = residual
        y = torch_port.allreduce_path_dist(x, w, self.eps).to(x.dtype)
        return self._plant(y, "residual" if residual is not None else "forward")

    def backward(self, dy, x, w):
        from oracle import torch_port

        dx, dw = torch_port.backward_dist(x, dy, w, self.eps)
        return self._plant(dx.to(x.dtype), "backward"), dw.to(w.dtype)

    def status(self):
        return {"code": 0}


def _workload():
    return dict(name="custom", hidden=512, rows=300, dtype=torch.bfloat16, eps=1e-6, seed_base=1000)


def _run_parity(world, rank, bad_rank, bad_what):
    w = _workload()
    wl = bench.load_workloads()
    hl = w["hidden"] // world
    x, wt = wl.make_slice(w["rows"], hl, w["dtype"], w["seed_base"] + rank)
    return bench.parity_check(_OracleModule(w["eps"], rank, bad_rank, bad_what), w, world, rank,
                              x, wt, n_sample=64)


@pytest.mark.parametrize("bad_what", [None, "forward", "residual", "backward"])
def test_parity_check_one_rank(bad_what):
    # the stand-in module's all_reduce needs a process group, here of one gloo rank
    dist.init_process_group("gloo", rank=0, world_size=1,
                            init_method=f"tcp://127.0.0.1:{bench.free_port()}")
    try:
        res = _run_parity(1, 0, 0 if bad_what else None, bad_what)
    finally:
        dist.destroy_process_group()
    assert res["ok"] == (bad_what is None), res
    assert set(res["checks"]) == {"forward", "residual", "backward"}
    if bad_what:
        assert not res["checks"][bad_what]["ok"]


def _gloo_worker(rank, world, port, bad_rank, bad_what, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = _run_parity(world, rank, bad_rank, bad_what)
        q.put((rank, res["ok"], res.get("checks")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad_rank,bad_what", [(None, None), (1, "forward"), (0, "backward")])
def test_parity_check_two_gloo_ranks(bad_rank, bad_what):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = bench.free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, bad_rank, bad_what, q))
             for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (ok, checks)) for r, ok, checks in (q.get(timeout=240) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = bad_what is None
    assert out[0][0] == want and out[1][0] == want       # every rank learns the verdict
    if bad_what:
        assert not out[0][1][bad_what]["ok"]
