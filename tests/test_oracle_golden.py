"""The CPU oracle against golden vectors made by the reference itself
(tests/golden/make_golden.py runs reference_tp_rmsnorm under gloo)."""
import numpy as np
import pytest

from conftest import load_golden
from oracle import tp_rmsnorm as O

CASES = sorted(load_golden().keys())


@pytest.mark.parametrize("name", CASES)
def test_allreduce_restatement_matches_reference(golden, name):
    c = golden[name]
    dt = c["meta"]["dtype"]
    outs = O.allreduce_path(c["x"], c["w"], c["meta"]["eps"], dt)
    for got, want in zip(outs, c["y"]):
        r = O.compare("f32", got, want)          # fp32 output: relative 1e-5
        assert r["ok"], r
        if dt != "f32":                          # rounded to x's dtype: bit-identical
            assert np.array_equal(O.from_f32(dt, got), O.from_f32(dt, want))


@pytest.mark.parametrize("name", [n for n in CASES if "overflow" not in n])
def test_fused_formula_within_tolerance_of_reference(golden, name):
    """The fused-kernel formula (fp32 squares, S / hidden) meets the parity bar
    against the reference's AllReduce output, compared in x's dtype."""
    c = golden[name]
    dt = c["meta"]["dtype"]
    outs = O.fused_path(c["x"], c["w"], c["meta"]["eps"], dt)
    for got, want in zip(outs, c["y"]):
        r = O.compare(dt, O.round_to(dt, got), O.round_to(dt, want))
        assert r["ok"], r


def test_fp16_overflow_divergence_is_confined_to_overflowing_rows(golden):
    """In fp16 the reference squares in fp16 (x.pow(2), bench_rmsnorm_tp.py:18):
    |x| >= 256 overflows to inf and the whole row comes out 0. The fused formula
    squares in fp32 and stays finite. They must agree on every other row."""
    c = golden["f16_tp2_overflow"]
    xs = [O.to_f32("f16", x) for x in c["x"]]
    overflow_rows = np.zeros(xs[0].shape[0], dtype=bool)
    for x in xs:
        overflow_rows |= (np.abs(x) >= 256.0).any(axis=1)
    assert overflow_rows.any() and not overflow_rows.all()
    fused = O.fused_path(c["x"], c["w"], c["meta"]["eps"], "f16")
    for got, want in zip(fused, c["y"]):
        assert np.all(want[overflow_rows] == 0.0)
        assert np.all(np.isfinite(got)) and np.any(got[overflow_rows] != 0.0)
        r = O.compare("f16", O.round_to("f16", got[~overflow_rows]),
                      O.round_to("f16", want[~overflow_rows]))
        assert r["ok"], r


def test_bf16_rounding_helpers_round_trip():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**16, size=4096, dtype=np.uint16)
    f = O.bf16_bits_to_f32(bits)
    finite = np.isfinite(f)
    assert np.array_equal(O.f32_to_bf16_bits(f)[finite], bits[finite])
    # ties round to even
    assert O.f32_to_bf16_bits(np.array([1.0 + 2**-8], np.float32))[0] == 0x3F80
    assert O.f32_to_bf16_bits(np.array([1.0 + 3 * 2**-8], np.float32))[0] == 0x3F82


def test_compare_flags_planted_error():
    """A mistake planted in the oracle's output is caught by the comparison."""
    c = load_golden()["bf16_tp2"]
    outs = O.allreduce_path(c["x"], c["w"], c["meta"]["eps"], "bf16")
    bad = outs[0].copy()
    bad[3, 5] *= 1.05
    assert not O.compare("bf16", O.round_to("bf16", bad), O.round_to("bf16", c["y"][0]))["ok"]
