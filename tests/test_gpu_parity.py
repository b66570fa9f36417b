"""GPU parity of the CUDA path against the CPU oracle (through the C-ABI).

* TP = 1 (local kernel) and emulated TP = 2/4/8 (every rank in one cooperative
  launch on one GPU) on the reference's golden vectors;
* the real forward entry point at TP = 2/4/8 on one GPU, with the other ranks'
  mailbox words written by the host (their pushes) and their mailboxes stood in
  for by device buffers (checked for our pushes);
* shape / dtype sweeps against the oracle; unaligned pointers (generic kernel);
* full-size configurations checked through size-independent properties and a
  sampled-row oracle comparison.
Tolerances (oracle.tp_rmsnorm.TOLERANCE): fp32 rtol 1e-5 (atol 1e-6); bf16/fp16
atol 1e-2 + rtol 1.6e-2 (one ulp of the output type).
"""
import numpy as np
import pytest
import torch

import rmsnorm_tp_b200 as rtp
from conftest import load_golden
from gpu_helpers import (TORCH_DTYPES, check_against_oracle, device_view, from_np, out_f32,
                         pack_slots, slot_index, to_np)
from oracle import tp_rmsnorm as O
from rmsnorm_tp_b200.workloads import BY_NAME, make_group

pytestmark = pytest.mark.gpu
GOLDEN = load_golden()


def _assert_ok(results, what=""):
    for r, res in enumerate(results):
        assert res["ok"], f"{what} rank {r}: {res}"


# --------------------------------------------------------------------------- golden
@pytest.mark.parametrize("name", sorted(n for n in GOLDEN if GOLDEN[n]["meta"]["tp"] == 1))
def test_local_kernel_on_reference_golden(name):
    c = GOLDEN[name]
    dt, eps = c["meta"]["dtype"], c["meta"]["eps"]
    x = from_np(dt, c["x"][0])
    w = from_np(dt, c["w"][0])
    y = rtp.local_rmsnorm(x, w, eps)
    torch.cuda.synchronize()
    res = O.compare(dt, out_f32(dt, y), O.round_to(dt, c["y"][0]))
    assert res["ok"], res


@pytest.mark.parametrize("name", sorted(n for n in GOLDEN if GOLDEN[n]["meta"]["tp"] > 1))
def test_emulated_group_on_reference_golden(name):
    c = GOLDEN[name]
    dt, eps, tp = c["meta"]["dtype"], c["meta"]["eps"], c["meta"]["tp"]
    g = rtp.EmulatedTPGroup(tp, eps=eps, num_max_rows=64, timeout_s=5.0)
    try:
        xs = [from_np(dt, x) for x in c["x"]]
        ws = [from_np(dt, w) for w in c["w"]]
        outs = g.forward(xs, ws)
        torch.cuda.synchronize()
        if "overflow" in name:
            # the reference's fp16 squares overflow there; parity is against the fused formula
            _assert_ok(check_against_oracle(dt, xs, ws, eps, outs, reference=False), name)
        else:
            for r in range(tp):
                res = O.compare(dt, out_f32(dt, outs[r]), O.round_to(dt, c["y"][r]))
                assert res["ok"], (r, res)
        for b in g.bufs:
            assert b.poll_error() == 0
    finally:
        g.destroy()


# --------------------------------------------------------------------------- sweeps
LOCAL_WIDTHS = [8, 37, 64, 96, 256, 384, 512, 1000, 1024, 2048, 3000, 4096, 8192, 16384, 32768]


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("hidden", LOCAL_WIDTHS)
@pytest.mark.parametrize("rows", [1, 3, 64, 257])
def test_local_kernel_sweep(family, dtype, hidden, rows):
    xs, ws = make_group(rows, hidden, 1, TORCH_DTYPES[dtype], 1000 + hidden + rows)
    x, w = xs[0].cuda(), ws[0].cuda()
    y = rtp.local_rmsnorm(x, w, 1e-6)
    torch.cuda.synchronize()
    _assert_ok(check_against_oracle(dtype, [x], [w], 1e-6, [y]), f"{dtype} {hidden} {rows}")


@pytest.mark.parametrize("tp", [2, 3, 4, 8])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("hl", [37, 64, 512, 1024, 2048, 4096])
@pytest.mark.parametrize("rows", [1, 7, 300])
def test_emulated_group_sweep(family, tp, dtype, hl, rows):
    xs, ws = make_group(rows, hl * tp, tp, TORCH_DTYPES[dtype], 7 * hl + rows)
    xs = [x.cuda() for x in xs]
    ws = [w.cuda() for w in ws]
    g = rtp.EmulatedTPGroup(tp, eps=1e-5, num_max_rows=512, timeout_s=5.0)
    try:
        for _ in range(2):  # both generation buffers
            outs = g.forward(xs, ws)
            torch.cuda.synchronize()
            _assert_ok(check_against_oracle(dtype, xs, ws, 1e-5, outs), f"tp{tp} {dtype} {hl} {rows}")
            # every rank normalised each row with the same inverse rms: rank-order sums are identical
            assert all(b.poll_error() == 0 for b in g.bufs)
        assert all(b.device_generation() == 2 for b in g.bufs)
    finally:
        g.destroy()


def test_unaligned_pointers_take_the_generic_kernel():
    xs, ws = make_group(33, 2 * 520, 2, torch.bfloat16, 5)
    # a one-element offset into a larger buffer breaks the 16-byte alignment
    xs_off = []
    for x in xs:
        big = torch.empty(x.numel() + 1, dtype=x.dtype, device="cuda")
        big[1:].copy_(x.flatten().cuda())
        xs_off.append(big[1:].view(x.shape))
    ws = [w.cuda() for w in ws]
    assert xs_off[0].data_ptr() % 16 != 0
    g = rtp.EmulatedTPGroup(2, eps=1e-6, num_max_rows=64, timeout_s=5.0)
    try:
        outs = g.forward(xs_off, ws)
        torch.cuda.synchronize()
        _assert_ok(check_against_oracle("bf16", xs_off, ws, 1e-6, outs))
    finally:
        g.destroy()
    y = rtp.local_rmsnorm(xs_off[0], ws[0], 1e-6)
    torch.cuda.synchronize()
    _assert_ok(check_against_oracle("bf16", [xs_off[0]], [ws[0]], 1e-6, [y]))


# --------------------------------------------------------------------------- real entry point
@pytest.mark.parametrize("tp,rank", [(2, 0), (2, 1), (4, 2), (8, 5)])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("hl,rows", [(1024, 1), (512, 77), (2048, 300), (4096, 5)])
def test_forward_entry_point_with_host_written_peer_slots(family, tp, rank, dtype, hl, rows):
    """rmsnorm_tp_forward at TP > 1 on one GPU. Before each call the host writes
    the other ranks' {partial, tag} words into this rank's mailbox, as their
    pushes would; the peers' mailboxes are device buffers that must receive
    this rank's partials with the call's tag."""
    nmax = 512
    buf = rtp.TPCommBuffer(rank, tp, nmax)
    buf.allocate()
    buf.set_timeout(5.0)
    box_ptr, box_bytes = buf.mailbox()
    mine = device_view(box_ptr, box_bytes)
    fakes = {}
    for q in range(tp):
        if q != rank:
            fakes[q] = torch.zeros(box_bytes // 8, dtype=torch.int64, device="cuda")
            buf.attach_peer(q, fakes[q].data_ptr())
    buf.finalize_setup()
    try:
        for call in range(3):
            xs, ws = make_group(rows, hl * tp, tp, TORCH_DTYPES[dtype], 100 * call + rows)
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
            # this rank's pushes: slot [b][rank][row] of every peer, with this call's tag
            lo = slot_index(b, rank, tp, nmax, 0)
            for q, f in fakes.items():
                words = f[lo:lo + rows].cpu().numpy().view(np.uint64)
                assert np.all((words >> np.uint64(32)) == tag)
                vals = (words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
                np.testing.assert_allclose(vals, partials[rank], rtol=2e-6)
        assert buf.device_generation() == 3
    finally:
        buf.destroy()


# --------------------------------------------------------------------------- full size
def _sampled_oracle_check(dtype, xs, ws, eps, outs, n=96, seed=0):
    rows = xs[0].shape[0]
    idx = np.sort(np.random.default_rng(seed).choice(rows, size=min(n, rows), replace=False))
    ti = torch.from_numpy(idx).to(xs[0].device)
    sub = lambda ts: [t.index_select(0, ti) for t in ts]  # noqa: E731
    _assert_ok(check_against_oracle(dtype, sub(xs), ws, eps, sub(outs)), f"sampled {dtype}")


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_llama3_8b_config_full_size(family, tp):
    cfg = BY_NAME["llama3_8b"]
    rows = cfg.rows[0]
    xs, ws = make_group(rows, cfg.hidden, tp, cfg.dtype, cfg.seed_base, device="cuda")
    if tp == 1:
        outs = [rtp.local_rmsnorm(xs[0], ws[0], cfg.eps)]
        outs2 = [rtp.local_rmsnorm(xs[0], ws[0], cfg.eps)]
    else:
        g = rtp.EmulatedTPGroup(tp, eps=cfg.eps, num_max_rows=rows, timeout_s=5.0)
        try:
            outs = g.forward(xs, ws)
            outs2 = g.forward(xs, ws)
            torch.cuda.synchronize()
        finally:
            g.destroy()
    torch.cuda.synchronize()
    _sampled_oracle_check("bf16", xs, ws, cfg.eps, outs)
    for a, b in zip(outs, outs2):  # deterministic: bit-identical across calls
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_rows_are_independent_permutation_equivariance():
    cfg = BY_NAME["decode_llama70b"]
    tp, rows = 8, 256
    xs, ws = make_group(rows, cfg.hidden, tp, cfg.dtype, 3, device="cuda")
    perm = torch.randperm(rows, generator=torch.Generator().manual_seed(1)).cuda()
    g = rtp.EmulatedTPGroup(tp, eps=cfg.eps, num_max_rows=rows, timeout_s=5.0)
    try:
        outs = g.forward(xs, ws)
        outs_p = g.forward([x[perm] for x in xs], ws)
        torch.cuda.synchronize()
    finally:
        g.destroy()
    for a, b in zip(outs, outs_p):
        assert torch.equal(a[perm].view(torch.int16), b.view(torch.int16))


def test_stress_pattern_zero_rows_and_outlier_channels(family):
    cfg = BY_NAME["stress"]
    tp, rows = 8, 4096
    xs, ws = make_group(rows, cfg.hidden, tp, cfg.dtype, cfg.seed_base, stress=True, device="cuda")
    zero_rows = torch.stack([(x == 0).all(dim=1) for x in xs]).all(dim=0)
    assert zero_rows.any()
    g = rtp.EmulatedTPGroup(tp, eps=cfg.eps, num_max_rows=rows, timeout_s=5.0)
    try:
        g.reset(2**32 - 3)   # start just below the 32-bit tag wrap
        for _ in range(6):
            outs = g.forward(xs, ws)
        torch.cuda.synchronize()
        assert all(b.device_generation() == 2**32 + 3 for b in g.bufs)
    finally:
        g.destroy()
    for y in outs:
        assert torch.isfinite(y.float()).all()
        assert (y[zero_rows] == 0).all()
    _sampled_oracle_check("bf16", xs, ws, cfg.eps, outs, n=128)


def test_generation_counter_at_its_top_and_every_grid_size(family):
    """The device counter advances by exactly one per forward launch and two per
    backward launch whatever the grid (row counts from 1 to many waves), up to
    the largest generation it holds; a larger reset is an argument error."""
    tp, hl = 2, 1024
    top = 2**44 - 1
    g = rtp.EmulatedTPGroup(tp, eps=1e-5, num_max_rows=70000, timeout_s=5.0)
    try:
        with pytest.raises(rtp.RMSNormTPError):
            g.bufs[0].reset(top + 1)
        g.reset(top - 20)
        n = 0
        for rows in (1, 7, 300, 4096, 70000, 1):
            xs, ws = make_group(rows, hl * tp, tp, torch.bfloat16, rows, device="cuda")
            outs = g.forward(xs, ws)
            n += 1
            torch.cuda.synchronize()
            _sampled_oracle_check("bf16", xs, ws, 1e-5, outs, n=min(rows, 64))
            assert all(b.device_generation() == top - 20 + n for b in g.bufs)
        dys = [torch.randn_like(x) for x in xs]
        g.backward(dys, xs, ws)
        torch.cuda.synchronize()
        assert all(b.device_generation() == top - 20 + n + 2 for b in g.bufs)
        assert all(b.status()["next_generation"] == top - 20 + n + 2 for b in g.bufs)
    finally:
        g.destroy()


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_prefill_config_full_size_tp8(family, dtype):
    cfg = BY_NAME["prefill"]
    tp, rows = 8, 65536
    xs, ws = make_group(rows, cfg.hidden, tp, TORCH_DTYPES[dtype], cfg.seed_base, device="cuda")
    g = rtp.EmulatedTPGroup(tp, eps=cfg.eps, num_max_rows=rows, timeout_s=5.0)
    try:
        outs = g.forward(xs, ws)
        torch.cuda.synchronize()
    finally:
        g.destroy()
    _sampled_oracle_check(dtype, xs, ws, cfg.eps, outs)
