"""World-size-2 gloo tests on CPU: the oracle's distributed form against the
reference's golden vectors, the bootstrap handle exchange, and a rank that never
joins the exchange (the other rank gets an error from the group timeout, no hang)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_golden


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _to_torch(dtype, a):
    if dtype == "bf16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _oracle_worker(rank, world, port, results):
    from oracle import torch_port

    _init(rank, world, port)
    try:
        golden = load_golden()
        out = {}
        for name in ("f32_tp2_cfg1", "bf16_tp2", "f16_tp2", "f32_tp2_ragged", "f16_tp2_overflow"):
            c = golden[name]
            dt = c["meta"]["dtype"]
            x = _to_torch(dt, c["x"][rank])
            w = _to_torch(dt, c["w"][rank])
            y = torch_port.allreduce_path_dist(x, w, c["meta"]["eps"])
            out[name] = bool(np.array_equal(y.float().numpy(), c["y"][rank]))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_gloo_allreduce_port_reproduces_reference_bit_exactly():
    port = _free_port()
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_oracle_worker, args=(2, port, results), nprocs=2, join=True)
        for r in range(2):
            assert all(results[r].values()), results[r]


def test_group_port_matches_dist_port():
    from oracle import torch_port

    c = load_golden()["bf16_tp4"]
    xs = [_to_torch("bf16", x) for x in c["x"]]
    ws = [_to_torch("bf16", w) for w in c["w"]]
    ys = torch_port.allreduce_path_group(xs, ws, c["meta"]["eps"])
    for y, want in zip(ys, c["y"]):
        np.testing.assert_allclose(y.float().numpy(), want, rtol=1e-6, atol=1e-7)


def _exchange_worker(rank, world, port, results):
    from rmsnorm_tp_b200 import IpcHandle, exchange_handles

    _init(rank, world, port)
    try:
        mine = IpcHandle(bytes([rank + 1]) * 128)
        devices, handles = exchange_handles(dist.group.WORLD, 10 + rank, mine)
        results[rank] = (devices, [h.to_bytes()[0] for h in handles])
    finally:
        dist.destroy_process_group()


def test_handle_exchange_over_gloo():
    port = _free_port()
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_exchange_worker, args=(2, port, results), nprocs=2, join=True)
        for r in range(2):
            assert results[r] == ([10, 11], [1, 2])


def _missing_peer_worker(rank, world, port, results):
    from rmsnorm_tp_b200 import IpcHandle, exchange_handles

    # the rendezvous waits as long as the ranks' start-up may take; only the
    # exchange runs over a group with a short timeout
    _init(rank, world, port)
    short = dist.new_group(ranks=[0, 1], timeout=datetime.timedelta(seconds=3))
    try:
        if rank == 1:
            results[rank] = "left"      # never joins the exchange
            return
        try:
            exchange_handles(short, 0, IpcHandle(b"\0" * 128))
            results[rank] = "no error"
        except Exception as e:          # the group timeout ends the wait
            results[rank] = type(e).__name__
    finally:
        pass


def test_rank_that_never_joins_produces_an_error_not_a_hang():
    port = _free_port()
    with mp.Manager() as m:
        results = m.dict()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_missing_peer_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        for p in procs:
            if p.is_alive():
                p.kill()
                pytest.fail("a rank hung")
        assert results[1] == "left"
        assert results[0] not in ("no error", None), results[0]


def _backward_worker(rank, world, port, results):
    from oracle import tp_rmsnorm as O
    from oracle import torch_port
    from rmsnorm_tp_b200.workloads import make_group

    _init(rank, world, port)
    try:
        xs, ws = make_group(24, 256 * world, world, torch.float32, 700)
        dys, _ = make_group(24, 256 * world, world, torch.float32, 800)
        dx, dw = torch_port.backward_dist(xs[rank], dys[rank], ws[rank], 1e-6)
        want_dx, want_dw = O.backward_path([x.numpy() for x in xs], [d.numpy() for d in dys],
                                           [w.numpy() for w in ws], 1e-6, "f32")
        results[rank] = (bool(np.allclose(dx.numpy(), want_dx[rank], rtol=1e-5, atol=1e-6)),
                         bool(np.allclose(dw.numpy(), want_dw[rank], rtol=1e-5, atol=1e-5)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_exchange_backward_matches_the_oracle():
    """The backward's two per-row exchanges, done by gloo all_reduce on two ranks,
    agree with the closed-form oracle on every rank's slice."""
    port = _free_port()
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_backward_worker, args=(2, port, results), nprocs=2, join=True)
        assert dict(results) == {0: (True, True), 1: (True, True)}
