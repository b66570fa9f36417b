"""Property tests of the oracle against torch on CPU, over random shapes, dtypes
and value scales (hypothesis): the numpy restatement of the reference's AllReduce
path against its torch port, the residual add against torch's own ``x + r``
(including overflow to inf), and the backward against autograd."""
import numpy as np
import torch
from hypothesis import given, settings, strategies as st

from gpu_helpers import NAMES, to_np
from oracle import tp_rmsnorm as O
from oracle import torch_port

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
SETTINGS = settings(max_examples=40, deadline=None)


def _group(rows, hl, tp, dtype, scale, seed):
    g = torch.Generator().manual_seed(seed)
    xs = [(torch.randn(rows, hl, generator=g) * scale).to(dtype) for _ in range(tp)]
    ws = [(1.0 + 0.1 * torch.randn(hl, generator=g)).to(dtype) for _ in range(tp)]
    return xs, ws


@SETTINGS
@given(rows=st.integers(1, 9), hl=st.integers(1, 70), tp=st.sampled_from([1, 2, 3, 4, 8]),
       dtype=st.sampled_from(DTYPES), scale=st.sampled_from([1e-3, 1.0, 30.0]),
       seed=st.integers(0, 2**31 - 1))
def test_allreduce_restatement_matches_the_torch_port(rows, hl, tp, dtype, scale, seed):
    name = NAMES[dtype]
    xs, ws = _group(rows, hl, tp, dtype, scale, seed)
    want = torch_port.allreduce_path_group(xs, ws, 1e-6)
    got = O.allreduce_path([to_np(x) for x in xs], [to_np(w) for w in ws], 1e-6, name)
    for g, t in zip(got, want):
        # rounded to x's dtype the two agree within the parity tolerance (float64
        # vs fp32 accumulation order of the means)
        r = O.compare(name, O.round_to(name, g), O.round_to(name, t.float().numpy()))
        assert r["ok"], r


@SETTINGS
@given(rows=st.integers(1, 6), hl=st.integers(1, 64), dtype=st.sampled_from(DTYPES),
       scale=st.sampled_from([1.0, 4e4, 2e38]), seed=st.integers(0, 2**31 - 1))
def test_residual_add_matches_torch_bit_exactly(rows, hl, dtype, scale, seed):
    name = NAMES[dtype]
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, hl, generator=g) * scale).to(dtype)
    r = (torch.randn(rows, hl, generator=g) * scale).to(dtype)
    got = np.asarray(O.residual_add(to_np(x), to_np(r), name))
    want = to_np(x + r)
    # NaN (inf + -inf) must match as NaN; its bit pattern is the platform's
    got_nan, want_nan = np.isnan(O.to_f32(name, got)), np.isnan(O.to_f32(name, want))
    np.testing.assert_array_equal(got_nan, want_nan)
    bits = np.uint32 if dtype == torch.float32 else np.uint16
    np.testing.assert_array_equal(got.view(bits)[~got_nan], want.view(bits)[~want_nan])


@SETTINGS
@given(rows=st.integers(1, 8), hl=st.integers(1, 48), tp=st.sampled_from([1, 2, 4]),
       dtype=st.sampled_from([torch.float32, torch.bfloat16]), seed=st.integers(0, 2**31 - 1))
def test_backward_matches_autograd(rows, hl, tp, dtype, seed):
    name = NAMES[dtype]
    xs, ws = _group(rows, hl, tp, dtype, 1.0, seed)
    dys, _ = _group(rows, hl, tp, dtype, 1.0, seed + 1)
    x64 = [x.double().requires_grad_() for x in xs]
    w64 = [w.double().requires_grad_() for w in ws]
    ys = torch_port.allreduce_path_group(x64, w64, 1e-6)
    sum((y * dy.double()).sum() for y, dy in zip(ys, dys)).backward()
    dxs, dws = O.backward_path([to_np(x) for x in xs], [to_np(d) for d in dys],
                               [to_np(w) for w in ws], 1e-6, name)
    # dx = inv * g - x * inv^3 * D / H can cancel to far below its two terms (a row
    # of one element cancels to ~eps / S of them); the reference formula computes
    # its variance in fp32 (mean(dtype=float32)) even for float64 inputs, so
    # autograd's dx carries fp32 rounding of the terms' size
    hidden = hl * tp
    X = [x.double().numpy() for x in xs]
    W = [w.double().numpy() for w in ws]
    DY = [d.double().numpy() for d in dys]
    S = sum((x * x).sum(axis=-1) for x in X)[..., None]
    D = sum((dy * w * x).sum(axis=-1) for x, dy, w in zip(X, DY, W))[..., None]
    inv = 1.0 / np.sqrt(S / hidden + 1e-6)
    for dx, dw, xt, wt, x, w, dy in zip(dxs, dws, x64, w64, X, W, DY):
        terms = np.abs(inv * dy * w) + np.abs(x * inv ** 3 * D / hidden)
        np.testing.assert_allclose(dx, xt.grad.numpy(), rtol=1e-5, atol=1e-6 + 4e-7 * terms.max())
        np.testing.assert_allclose(dw, wt.grad.numpy(), rtol=1e-5, atol=1e-6)
