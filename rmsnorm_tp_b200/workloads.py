"""Seeded synthetic inputs of the benchmark configurations.

There is no public dataset for this path; every configuration draws
x ~ N(0, 1) and weight ~ 1 + 0.1 * N(0, 1) per rank slice from a torch
generator seeded with ``seed_base + rank``, then casts to the working dtype.
The stress configuration additionally scales 1% of the channels by 100 and
zeroes 1% of the rows (the same rows on every rank, so those rows are zero
across the whole hidden dimension).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Tuple

import torch

DTYPE_NAMES = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}
NAME_DTYPES = {v: k for k, v in DTYPE_NAMES.items()}


@dataclass(frozen=True)
class Config:
    name: str
    hidden: int
    dtype: torch.dtype
    eps: float
    seed_base: int
    rows: Tuple[int, ...]
    tps: Tuple[int, ...]
    stress: bool = False
    note: str = field(default="", compare=False)


# The five configurations of the benchmark (index = position in its list).
CONFIGS = (
    Config("cpu_gloo_tp2", 4096, torch.float32, 1e-6, 0, (1024,), (2,),
           note="CPU/gloo reference path, world_size 2"),
    Config("llama3_8b", 4096, torch.bfloat16, 1e-6, 1000, (4096,), (1, 2, 4, 8),
           note="Llama-3-8B-shaped rows, TP = 1/2/4/8"),
    Config("decode_llama70b", 8192, torch.bfloat16, 1e-5, 1000,
           (1, 2, 4, 8, 16, 32, 64, 128, 256), (8,), note="decode latency sweep"),
    Config("prefill", 8192, torch.bfloat16, 1e-5, 1000, (8192, 16384, 32768, 65536), (2, 4, 8),
           note="prefill throughput sweep (bf16 and fp16)"),
    Config("stress", 16384, torch.bfloat16, 1e-5, 1000, (65536,), (8,), stress=True,
           note="outlier channels, zero rows, many calls with launch skew"),
)
BY_NAME = {c.name: c for c in CONFIGS}


def make_slice(rows: int, local_hidden: int, dtype: torch.dtype, seed: int, *,
               stress: bool = False, stress_seed: int = 0,
               device: str = "cpu") -> Tuple[torch.Tensor, torch.Tensor]:
    """One rank's (x [rows, local_hidden], weight [local_hidden]) in `dtype`.

    Generated in fp32 on `device` from a generator seeded with `seed`; the
    stress pattern (channel outliers chosen per rank from `seed`, zero rows
    chosen from `stress_seed`, shared by every rank) is applied before the cast.
    """
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, local_hidden, generator=g, device=device, dtype=torch.float32)
    w = 1.0 + 0.1 * torch.randn(local_hidden, generator=g, device=device, dtype=torch.float32)
    if stress:
        n_ch = max(1, round(0.01 * local_hidden))
        ch = torch.randperm(local_hidden, generator=g, device=device)[:n_ch]
        x[:, ch] *= 100.0
        gz = torch.Generator(device=device).manual_seed(stress_seed)
        n_rows = max(1, round(0.01 * rows))
        zr = torch.randperm(rows, generator=gz, device=device)[:n_rows]
        x[zr, :] = 0.0
    return x.to(dtype), w.to(dtype)


def make_group(rows: int, hidden: int, tp: int, dtype: torch.dtype, seed_base: int, *,
               stress: bool = False, device: str = "cpu"):
    """Every rank's slice of one call: lists xs[tp], ws[tp]."""
    if hidden % tp:
        raise ValueError(f"hidden {hidden} is not divisible by tp {tp}")
    hl = hidden // tp
    xs, ws = [], []
    for r in range(tp):
        x, w = make_slice(rows, hl, dtype, seed_base + r, stress=stress, stress_seed=seed_base,
                          device=device)
        xs.append(x)
        ws.append(w)
    return xs, ws


def algorithmic_bytes(rows: int, local_hidden: int, dtype: torch.dtype) -> int:
    """HBM bytes one rank must move per call: read x, write y, read the weight once."""
    s = torch.tensor([], dtype=dtype).element_size()
    return 2 * rows * local_hidden * s + local_hidden * s


def make_linear_group(rows: int, k_local: int, hidden: int, tp: int, dtype: torch.dtype,
                      seed: int, *, device: str = "cpu"):
    """Inputs of the fused row-parallel linear for every rank: a_r [rows, k_local]
    ~ N(0, 1), the linear weight slice lw_r [hidden, k_local] ~ N(0, 1 / (k_local * tp))
    (unit-variance outputs after the sum over ranks), and the norm weight slice
    g_r [hidden / tp] ~ 1 + 0.1 N(0, 1); each rank from a generator seeded seed + rank."""
    if hidden % tp:
        raise ValueError(f"hidden {hidden} is not divisible by tp {tp}")
    as_, lws, gs = [], [], []
    scale = (k_local * tp) ** -0.5
    for r in range(tp):
        g = torch.Generator(device=device).manual_seed(seed + r)
        a = torch.randn(rows, k_local, generator=g, device=device, dtype=torch.float32)
        w = scale * torch.randn(hidden, k_local, generator=g, device=device, dtype=torch.float32)
        gm = 1.0 + 0.1 * torch.randn(hidden // tp, generator=g, device=device, dtype=torch.float32)
        as_.append(a.to(dtype))
        lws.append(w.to(dtype))
        gs.append(gm.to(dtype))
    return as_, lws, gs
