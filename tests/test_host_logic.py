"""Host-side logic without a GPU: generation arithmetic, launch plan and
row -> team coverage, the Python surface's contract checks, handle format,
and the C++ protocol test of the shared header."""
import os
import subprocess

import pytest
import torch

import rmsnorm_tp_b200 as rtp
from conftest import ROOT
from rmsnorm_tp_b200 import FusedTPRMSNorm, IpcHandle


def test_tags_never_zero_and_change_every_two_calls():
    for g0 in (0, 2**32 - 5, 2**32 - 1 - 5, 2 * (2**32 - 1) - 5, 2**40):
        for g in range(g0, g0 + 12):
            assert rtp.tag_of(g) != 0
            assert rtp.tag_of(g) != rtp.tag_of(g + 2)
            assert rtp.buffer_of(g) == g & 1
    assert rtp.tag_of(2**32 - 2) == 2**32 - 1 and rtp.tag_of(2**32 - 1) == 1


@pytest.fixture
def register_family():
    rtp.set_kernel_family("register")
    yield
    rtp.set_kernel_family("auto")


@pytest.mark.parametrize("tp", [1, 2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hl", [8, 64, 96, 256, 512, 1000, 1024, 2048, 4096, 8192, 16384, 32768, 65536])
def test_register_plan_capacity(register_family, dtype, hl, tp):
    es = torch.tensor([], dtype=dtype).element_size()
    p = rtp.plan(100, hl, dtype, tp=tp)
    if (hl * es) % 16 or hl * es // 16 > 2048:
        assert p["variant"] == -1 and p["depth"] == 1
    else:
        V = hl * es // 16
        if tp == 1:                                   # no exchange: every buffer loading
            assert 200 <= p["variant"] < 300 and p["depth"] in (3, 4, 6)
        else:                                         # 2 buffers loading + 1 awaiting peers
            assert 0 <= p["variant"] < 100 and p["depth"] == 3
        assert 32 * p["team_warps"] * p["vec_per_lane"] >= V            # whole row in registers
        assert p["rows_per_tile"] * 8 <= 32                               # one lane per (row, rank)
        assert p["vec_per_lane"] * p["rows_per_tile"] <= 4                # 3 tiles in flight fit
    assert p["block_threads"] % (32 * p["team_warps"]) == 0


@pytest.fixture
def bulk_family():
    rtp.set_kernel_family("bulk")
    yield
    rtp.set_kernel_family("auto")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hl", [8, 64, 96, 256, 512, 1000, 1024, 2048, 4096, 8192, 16384])
@pytest.mark.parametrize("tp", [1, 2, 3, 4, 8])
def test_bulk_plan_for_large_calls(dtype, hl, tp):
    es = torch.tensor([], dtype=dtype).element_size()
    row = hl * es
    if tp == 1:
        # >= 256 MiB of x at TP = 1: the automatic choice is bulk; one row less: register
        rows = -(-(256 << 20) // row)
        p = rtp.plan(rows, hl, dtype, tp=tp)
        below = rtp.plan(rows - 1, hl, dtype, tp=tp)
        assert not 100 <= below["variant"] < 200
        if row % 16 or row >= 16384:
            assert p["variant"] < 100 or p["variant"] >= 200
            return
    else:
        # with an exchange the bulk kernels run when forced
        rtp.set_kernel_family("bulk")
        try:
            p = rtp.plan(1 << 16, hl, dtype, tp=tp)
        finally:
            rtp.set_kernel_family("auto")
        if row % 16 or row > 16384:
            assert p["variant"] < 100 or p["variant"] >= 200
            return
    assert 100 <= p["variant"] < 200 and p["team_warps"] == 1 and p["depth"] == 3
    assert p["teams_per_cta"] == p["block_threads"] // 32 in (4, 8, 16)
    assert 1 <= p["rows_per_tile"] <= (32 // tp if tp > 1 else 32)       # one exchange round
    stages = p["vec_per_lane"]
    stage = -(-p["rows_per_tile"] * row // 128) * 128
    smem = -(-row // 128) * 128 + p["teams_per_cta"] * stages * stage
    assert smem <= 216 * 1024                                             # fits one CTA per SM


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hl", [8, 64, 96, 256, 512, 1000, 1024, 2048, 4096, 8192, 16384])
@pytest.mark.parametrize("tp", [2, 3, 4, 8])
@pytest.mark.parametrize("rows", [1, 7, 256, 4096, 65536])
def test_batch_plan_with_an_exchange(dtype, hl, tp, rows):
    """Aligned rows of up to 16 KB with an exchange take the batch kernels (when that
    family is chosen): batches
    of at most 32 rows (one lane per row in the exchange), a ring of at least 3
    slots in the shared-memory budget of 2 CTAs per SM, a grid of at most one
    resident wave."""
    es = torch.tensor([], dtype=dtype).element_size()
    row = hl * es
    rtp.set_kernel_family("batch")
    try:
        p = rtp.plan(rows, hl, dtype, tp=tp, resident_ctas=296)
    finally:
        rtp.set_kernel_family("auto")
    if row % 16 or row > 16384:
        assert not 500 <= p["variant"] < 600
        return
    assert p["variant"] == 500 and p["block_threads"] == 256 and p["teams_per_cta"] == 1
    bR, slots = p["rows_per_tile"], p["depth"]
    assert 1 <= bR <= 32 and bR * row <= max(16384, row)
    assert 3 <= slots <= 8 and p["vec_per_lane"] == slots
    slot = -(-bR * row // 128) * 128
    assert -(-row // 128) * 128 + slots * slot <= 100 * 1024               # 2 CTAs per SM
    assert p["tiles"] == -(-rows // bR) and p["grid"] == min(296, p["tiles"])
    if rows >= 2 * 296 * 32:
        assert bR == min(32, max(1, 16384 // row))                        # no needless shrinking


def test_unaligned_pointers_use_generic_kernel():
    assert rtp.plan(10, 1024, torch.bfloat16, aligned=False)["variant"] == -1


def test_kernel_family_switch():
    assert rtp.get_kernel_family() == "auto"
    bulk, batch = range(100, 200), range(500, 600)
    resident = range(600, 700)
    assert rtp.plan(10, 1024, torch.bfloat16)["variant"] >= 200          # small call: register (TP 1)
    assert rtp.plan(10, 1024, torch.bfloat16, tp=2)["variant"] in resident   # with an exchange
    assert rtp.plan(256, 2048, torch.bfloat16, tp=2)["variant"] in resident   # decode sizes
    assert rtp.plan(4096, 2048, torch.bfloat16, tp=2)["variant"] < 100  # the bench call at N=2: rotating
    assert rtp.plan(65536, 1024, torch.bfloat16, tp=2)["variant"] in bulk    # 128 MiB: bulk
    assert rtp.plan(10, 1000, torch.float32, tp=2)["variant"] in resident    # 4000-byte rows
    assert rtp.plan(10, 16384, torch.float32, tp=2)["variant"] == -1         # 64 KB rows: generic
    # more tiles than 4 per team: the rotating register kernel
    assert rtp.plan(6000, 2048, torch.bfloat16, tp=2, resident_ctas=296)["variant"] < 100
    assert rtp.plan(65536, 1024, torch.bfloat16)["variant"] >= 200         # 128 MiB, TP 1: local
    assert rtp.plan(262144, 1024, torch.bfloat16)["variant"] in bulk        # 512 MiB, TP 1: bulk
    rtp.set_kernel_family("register")
    try:
        assert rtp.plan(65536, 1024, torch.bfloat16)["variant"] >= 200
        assert rtp.plan(65536, 1024, torch.bfloat16, tp=4)["variant"] < 100
        rtp.set_kernel_family("bulk")
        assert rtp.plan(10, 1024, torch.bfloat16)["variant"] in bulk
        assert rtp.plan(10, 1024, torch.bfloat16, tp=4)["variant"] in bulk
        rtp.set_kernel_family("batch")
        assert rtp.plan(10, 1024, torch.bfloat16)["variant"] in batch      # TP 1 too when forced
        assert rtp.plan(10, 1024, torch.bfloat16, tp=8)["variant"] in batch
    finally:
        rtp.set_kernel_family("auto")


def test_push_mode_switch():
    assert rtp.get_push_mode() == "packed"
    try:
        rtp.set_push_mode("release")
        assert rtp.get_push_mode() == "release"
    finally:
        rtp.set_push_mode("packed")
    from rmsnorm_tp_b200 import _lib
    assert _lib.LIB.rmsnorm_tp_set_push_mode(2) == _lib.ERR_INVALID
    assert rtp.get_push_mode() == "packed"


@pytest.mark.parametrize("family", ["auto", "batch", "register"])
@pytest.mark.parametrize("rows", [0, 1, 2, 3, 7, 255, 256, 1000, 4097, 65536])
@pytest.mark.parametrize("hl", [64, 1024, 4096, 37])
@pytest.mark.parametrize("resident", [1, 7, 148, 1184])
@pytest.mark.parametrize("tp", [1, 3, 8])
def test_every_row_is_visited_exactly_once(rows, hl, resident, tp, family):
    rtp.set_kernel_family(family)
    try:
        p = rtp.plan(rows, hl, torch.bfloat16, tp=tp, resident_ctas=resident)
    finally:
        rtp.set_kernel_family("auto")
    assert p["grid"] <= max(1, resident)
    counts = rtp.plan_coverage(p, rows)
    assert len(counts) == rows and all(c == 1 for c in counts)


def test_grid_never_exceeds_one_resident_wave():
    p = rtp.plan(65536, 1024, torch.bfloat16, tp=8, resident_ctas=148)
    assert p["grid"] == 148 and p["tiles"] == 65536 // p["rows_per_tile"]
    p = rtp.plan(3, 1024, torch.bfloat16, tp=8, resident_ctas=148)
    assert p["grid"] == 1                                # a tiny call: one CTA


def test_tp1_module_keeps_reference_attributes():
    m = FusedTPRMSNorm(hidden_dim=4096, eps=1e-5)
    assert (m.tp_size, m.rank, m.eps, m.hidden_dim, m.num_max_rows) == (1, 0, 1e-5, 4096, 65536)
    assert m.comm_buf is None
    m.destroy()


def test_forward_contract_checks_raise_assertion_error():
    m = FusedTPRMSNorm(hidden_dim=64)
    x = torch.randn(4, 64)
    w = torch.randn(64)
    with pytest.raises(AssertionError):                  # not contiguous
        m.forward(x.t(), w)
    with pytest.raises(AssertionError):                  # unsupported dtype
        m.forward(x.double(), w.double())
    with pytest.raises(AssertionError):                  # mismatched dtypes
        m.forward(x, w.half())
    with pytest.raises(AssertionError):                  # weight shape
        m.forward(x, torch.randn(63))
    with pytest.raises(AssertionError):                  # CPU tensors: no CPU fallback
        m.forward(x, w)


def test_ipc_handle_bytes():
    with pytest.raises(RuntimeError, match="Invalid handle size"):
        IpcHandle().from_bytes(b"\0" * 127)
    raw = bytearray(128)
    raw[88:96] = (123456).to_bytes(8, "little")
    h = IpcHandle().from_bytes(bytes(raw))
    assert h.to_bytes() == bytes(raw) and h.alloc_size == 123456


def test_protocol_host_program(tmp_path):
    """Compile and run tests/cpp/test_protocol.cpp against the kernels' header."""
    exe = tmp_path / "test_protocol"
    src = os.path.join(ROOT, "tests", "cpp", "test_protocol.cpp")
    inc = os.path.join(ROOT, "rmsnorm_tp_b200", "csrc")
    subprocess.run(["g++", "-O2", "-std=c++17", "-pthread", "-Wall", "-I", inc, src, "-o", str(exe)],
                   check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "ALL PASS" in res.stdout


def _build_generation_program(tmp_path, *defines):
    exe = tmp_path / ("test_generation" + "".join(d.lower() for d in defines))
    src = os.path.join(ROOT, "tests", "cpp", "test_generation.cpp")
    inc = os.path.join(ROOT, "rmsnorm_tp_b200", "csrc")
    subprocess.run(["g++", "-O2", "-std=c++17", "-pthread", "-Wall", *[f"-D{d}" for d in defines],
                    "-I", inc, src, "-o", str(exe)], check=True)
    return exe


def test_generation_counter_host_program(tmp_path):
    """The device generation counter (shares of one-generation launches, the
    last CTA's store for two-generation ones) played by threads over launches of
    random grid sizes, orders and delays: every CTA reads its launch's generation
    and every launch advances the counter by exactly its step."""
    res = subprocess.run([str(_build_generation_program(tmp_path))], capture_output=True,
                         text=True, timeout=300)
    assert res.returncode == 0 and "ALL PASS" in res.stdout, res.stdout + res.stderr


def test_generation_counter_simulation_catches_an_advance_before_the_read(tmp_path):
    """Negative control: a CTA that advances the counter before reading it lets
    the launch's last CTA read the next generation -- the program must fail."""
    exe = _build_generation_program(tmp_path, "RTP_PLANT_ADD_BEFORE_READ")
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode != 0 and "FAIL" in res.stdout, res.stdout


def test_protocol_simulation_catches_an_early_second_push(tmp_path):
    """Negative control of the mixed forward / backward simulation: pushing a
    backward call's second partial before the row's first exchange completes lets
    a fast rank overwrite slots a slow rank still awaits -- the program must fail."""
    exe = tmp_path / "test_protocol_planted"
    src = os.path.join(ROOT, "tests", "cpp", "test_protocol.cpp")
    inc = os.path.join(ROOT, "rmsnorm_tp_b200", "csrc")
    subprocess.run(["g++", "-O2", "-std=c++17", "-pthread", "-Wall", "-DRTP_PLANT_EARLY_SECOND_PUSH",
                    "-I", inc, src, "-o", str(exe)], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode != 0 and "FAIL" in res.stdout, res.stdout


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("hl", [64, 512, 1000, 1024, 2048, 4096, 8192])
@pytest.mark.parametrize("rows", [1, 300, 4096, 9000])
def test_resident_plan_holds_at_most_four_tiles_per_team(tp, hl, rows):
    """With an exchange, a register plan of at most 256 rows whose teams would
    hold at most 4 tiles each runs the resident register kernel (every tile's
    loads in flight at once; its depth is the tiles per team); larger calls keep
    the rotating kernel."""
    p = rtp.plan(rows, hl, torch.float32, tp=tp, resident_ctas=296)
    teams = 296 * p["teams_per_cta"]
    if 600 <= p["variant"] < 700:
        assert rows <= 256
        assert p["tiles"] <= teams * 4 and p["depth"] == -(-p["tiles"] // teams)
        assert p["grid"] == min(296, -(-p["tiles"] // p["teams_per_cta"]))
    elif 0 <= p["variant"] < 100:
        assert p["tiles"] > teams * 4 or rows > 256


def test_profile_summary_means():
    """profile_summary turns the 20 in-kernel counters into means: waits per slow
    poll, launch span per launch, gap per counted gap, CTA figures per CTA; a
    counter that was never counted gives None, and the start-of-launch scratch
    value (UINT64_MAX as int64 -1) does not leak into any figure."""
    c = [0] * rtp.PROFILE_COUNTERS
    c[0], c[1], c[2] = 3_000, 2, 6              # 2 slow polls waiting 3 us in all, 6 fast
    c[3], c[4] = 1_000, 9_000
    c[5], c[6], c[7] = 8_000, 4_000, 4          # 4 CTAs with the pushed mark
    c[8], c[9] = 24_000, 4                      # 4 CTAs, 6 us each
    c[10], c[11] = 20_000, 2                    # 2 launches of 10 us
    c[12], c[13] = 1_500, 1                     # one gap of 1.5 us
    c[14] = -1
    c[17], c[18] = 6_000, 2                     # CTA start delays after the previous launch
    s = rtp.profile_summary(c)
    assert s["polls"] == 8 and s["slow_poll_share"] == 0.25 and s["mean_wait_us"] == 1.5
    assert s["launch_span_us"] == 10.0 and s["launch_gap_us"] == 1.5
    assert s["cta_us"] == 6.0 and s["cta_start_delay_us"] == 3.0
    assert s["cta_load_reduce_push_us"] == 2.0 and s["cta_poll_store_us"] == 1.0
    empty = rtp.profile_summary([0] * rtp.PROFILE_COUNTERS)
    assert empty["launch_gap_us"] is None and empty["cta_us"] is None and empty["polls"] == 0
