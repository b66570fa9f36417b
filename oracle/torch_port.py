"""torch-CPU port of the reference's AllReduce TP RMSNorm (test oracle / CPU baseline).

The reference path (bench_rmsnorm_tp.py:16-22) is a handful of torch ops around
an all_reduce; this module restates those ops so they can run where the
reference cannot travel:

* ``allreduce_path_group`` -- one process holds every rank's slice and the
  all_reduce becomes an in-process sum in rank order (what bench.py times as
  the CPU baseline, with all host threads);
* ``allreduce_path_dist`` -- one slice per process, the all_reduce done by
  torch.distributed (gloo on CPU in the multi-process tests).

The steps must match the reference's op for op (x.pow(2) in x's dtype, mean
with dtype=float32, SUM then divide by tp, x * rsqrt(v + eps) * w), because
that arithmetic is what parity is measured against.
"""
from __future__ import annotations

from typing import List, Sequence

import torch
import torch.distributed as dist


def _local_variance(x: torch.Tensor) -> torch.Tensor:
    # bench_rmsnorm_tp.py:18
    return x.pow(2).mean(dim=-1, keepdim=True, dtype=torch.float32)


def allreduce_path_group(xs: Sequence[torch.Tensor], ws: Sequence[torch.Tensor],
                         eps: float) -> List[torch.Tensor]:
    """Every rank's output of the AllReduce path, computed in one process."""
    tp = len(xs)
    total = _local_variance(xs[0])
    for x in xs[1:]:
        total = total + _local_variance(x)           # all_reduce SUM (:20)
    variance = total / tp if tp > 1 else total      # (:21)
    inv = torch.rsqrt(variance + eps)               # (:22)
    return [x * inv * w for x, w in zip(xs, ws)]


def allreduce_path_dist(x: torch.Tensor, w: torch.Tensor, eps: float, group=None) -> torch.Tensor:
    """This rank's output of the AllReduce path, the all_reduce done by torch.distributed."""
    tp = dist.get_world_size(group)
    variance = _local_variance(x)
    if tp > 1:
        dist.all_reduce(variance, op=dist.ReduceOp.SUM, group=group)   # (:20)
        variance = variance / tp                                       # (:21)
    return x * torch.rsqrt(variance + eps) * w                         # (:22)


def backward_dist(x: torch.Tensor, dy: torch.Tensor, w: torch.Tensor, eps: float, group=None):
    """This rank's (dx, dw) of the TP RMSNorm, the two per-row sums exchanged by
    torch.distributed all_reduce (gloo on CPU in the multi-process tests). The
    reference is forward-only; this restates the two-exchange backward of this
    repository's kernel (S = sum x^2 over the group, then D = sum dy*w*x over the
    group) in fp32 torch ops, as the derivative of bench_rmsnorm_tp.py:16-22."""
    tp = dist.get_world_size(group)
    hidden = x.shape[-1] * tp
    xf, dyf, wf = x.float(), dy.float(), w.float()
    S = (xf * xf).sum(dim=-1, keepdim=True)
    if tp > 1:
        dist.all_reduce(S, op=dist.ReduceOp.SUM, group=group)
    g = dyf * wf
    D = (g * xf).sum(dim=-1, keepdim=True)
    if tp > 1:
        dist.all_reduce(D, op=dist.ReduceOp.SUM, group=group)
    inv = torch.rsqrt(S / hidden + eps)
    dx = inv * g - xf * (inv ** 3) * (D / hidden)
    dw = (dyf * xf * inv).sum(dim=0)
    return dx, dw


def linear_rs_norm_group(as_: Sequence[torch.Tensor], lws: Sequence[torch.Tensor],
                         gammas: Sequence[torch.Tensor], eps: float,
                         residuals: Sequence[torch.Tensor] = None) -> List[torch.Tensor]:
    """The unfused pipeline of a Megatron-style block, every rank in one process:
    rank r's partial a_r @ lw_r^T (fp32 GEMM, rounded to the dtype as a reduce-scatter
    in that dtype receives it), the sum of every rank's column block in rank order,
    the residual add, then the reference's AllReduce TP RMSNorm
    (bench_rmsnorm_tp.py:16-22)."""
    tp = len(as_)
    dt = as_[0].dtype
    partials = [(a.float() @ w.float().t()).to(dt) for a, w in zip(as_, lws)]
    hl = partials[0].shape[1] // tp
    xs = []
    for o in range(tp):
        acc = partials[0][:, o * hl:(o + 1) * hl].float()
        for p in partials[1:]:
            acc = acc + p[:, o * hl:(o + 1) * hl].float()
        xs.append(acc.to(dt))
    if residuals is not None:
        xs = [(x.float() + r.float()).to(dt) for x, r in zip(xs, residuals)]
    return allreduce_path_group(xs, gammas, eps)
