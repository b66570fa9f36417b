"""Python surface of the fused TP RMSNorm, mirroring the reference's
``rmsnorm_tp`` package (rmsnorm_tp/__init__.py:1-135): ``FusedTPRMSNorm``,
``TPCommBuffer`` and ``IpcHandle`` keep their names, arguments and error
behaviour (``AssertionError`` for the contract checks the reference asserts,
``RuntimeError`` subclasses for native failures). Every compute call goes to
the C-ABI library; there is no torch or CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib
from ._lib import LIB, check

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}

try:  # fast path: the raw cudaStream_t of the current stream as an int
    _raw_stream = torch._C._cuda_getCurrentRawStream  # type: ignore[attr-defined]
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream_of(device_index: int) -> int:
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise AssertionError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16")


def _check_operands(x: torch.Tensor, weight: torch.Tensor) -> None:
    # reference rmsnorm_tp/__init__.py:96-97 asserts contiguity and dtype
    if not (x.is_contiguous() and weight.is_contiguous()):
        raise AssertionError("x and weight must be contiguous")
    if x.dtype not in _DTYPES or weight.dtype != x.dtype:
        raise AssertionError(
            f"x and weight must share one of float32/bfloat16/float16 (got {x.dtype}, {weight.dtype})"
        )
    if x.dim() != 2:
        raise AssertionError(f"x must be [num_rows, local_hidden_dim], got shape {tuple(x.shape)}")
    if weight.dim() != 1 or weight.shape[0] != x.shape[1]:
        raise AssertionError(
            f"weight must be [local_hidden_dim={x.shape[1]}], got shape {tuple(weight.shape)}"
        )
    if not (x.is_cuda and weight.is_cuda) or x.device != weight.device:
        raise AssertionError("x and weight must be CUDA tensors on the same device")


def _check_like(name: str, t: torch.Tensor, x: torch.Tensor) -> None:
    if t.shape != x.shape or t.dtype != x.dtype or t.device != x.device or not t.is_contiguous():
        raise AssertionError(f"{name} must be contiguous with x's shape, dtype and device")


def local_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                  out: Optional[torch.Tensor] = None,
                  residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """TP = 1 RMSNorm on the GPU: ``x * rsqrt(mean(x^2) + eps) * weight`` in fp32,
    rounded once to ``x.dtype`` (reference rmsnorm_tp/__init__.py:103-107).

    ``residual`` (optional, not in the reference): fused residual add in the same
    kernel -- ``z = x + residual`` (rounded to x's dtype) is written back into
    ``residual`` and normalised instead of x."""
    _check_operands(x, weight)
    if out is None:
        out = torch.empty_like(x)
    rows, hidden = x.shape
    if residual is not None:
        _check_like("residual", residual, x)
        check(
            LIB.rmsnorm_local_forward_residual(out.data_ptr(), residual.data_ptr(), x.data_ptr(),
                                               weight.data_ptr(), rows, hidden, _DTYPES[x.dtype],
                                               float(eps), _stream_of(x.device.index)),
            "rmsnorm_local_forward_residual",
        )
        return out
    check(
        LIB.rmsnorm_local_forward(out.data_ptr(), x.data_ptr(), weight.data_ptr(), rows, hidden,
                                  _DTYPES[x.dtype], float(eps), _stream_of(x.device.index)),
        "rmsnorm_local_forward",
    )
    return out


def _backward_operands(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor):
    _check_operands(x, weight)
    _check_like("dy", dy, x)
    dx = torch.empty_like(x)
    dw = torch.empty_like(weight)
    rows, hl = x.shape
    nbytes = LIB.rmsnorm_tp_backward_workspace_bytes(rows, hl)
    ws = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=x.device)
    return dx, dw, ws, nbytes


def local_rmsnorm_backward(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                           eps: float = 1e-6):
    """Gradients (dx, dw) of ``local_rmsnorm(x, weight, eps)`` for the output gradient dy
    (no reference counterpart: the reference is forward-only)."""
    dx, dw, ws, nbytes = _backward_operands(dy, x, weight)
    rows, hidden = x.shape
    check(
        LIB.rmsnorm_local_backward(dx.data_ptr(), dw.data_ptr(), dy.data_ptr(), x.data_ptr(),
                                   weight.data_ptr(), rows, hidden, _DTYPES[x.dtype], float(eps),
                                   ws.data_ptr(), nbytes, _stream_of(x.device.index)),
        "rmsnorm_local_backward",
    )
    return dx, dw


class IpcHandle:
    """Serialised mailbox handle (128 bytes), the counterpart of the reference's
    ``IpcHandle`` POD with ``to_bytes``/``from_bytes`` (csrc/common.hpp:13-16,
    csrc/bindings.cpp:151-162)."""

    SIZE = _lib.HANDLE_BYTES

    def __init__(self, data: bytes = b""):
        self._data = bytes(data)

    def to_bytes(self) -> bytes:
        return self._data

    def from_bytes(self, b: bytes) -> "IpcHandle":
        if len(b) != self.SIZE:  # reference bindings.cpp:159-160
            raise RuntimeError("Invalid handle size")
        self._data = bytes(b)
        return self

    @property
    def alloc_size(self) -> int:
        """Mailbox bytes recorded in the handle (reference IpcHandle.alloc_size)."""
        if len(self._data) != self.SIZE:
            return 0
        return int.from_bytes(self._data[88:96], "little")


class TPCommBuffer:
    """Per-rank mailbox for the TP group (reference rmsnorm_tp/__init__.py:6-37).

    The mailbox is u64 slot[2][tp_size][num_max_rows] in this rank's HBM, each
    slot one {fp32 partial sum of squares, 32-bit tag} word that peers write over
    NVLink. The generation counter lives on the device and the kernel advances
    it; ``generation`` here is a host-side count of launches kept for the
    reference's API.
    """

    def __init__(self, rank: int, tp_size: int, num_max_rows: int, device: Optional[int] = None,
                 linear_hidden: int = 0):
        self.rank = rank
        self.tp_size = tp_size
        self.num_max_rows = num_max_rows
        self.device = torch.cuda.current_device() if device is None else int(device)
        # > 0: the mailbox allocation also holds the receive buffer of the fused
        # row-parallel linear for this hidden width (FusedTPLinearRMSNorm)
        self.linear_hidden = int(linear_hidden)
        self._comm = ctypes.c_void_p()
        self._generation = 0

    # -- lifecycle (reference order: allocate, get_ipc_handle, open_remote_handle, finalize_setup)
    def allocate(self) -> None:
        if self._comm.value:
            raise RuntimeError("TPCommBuffer.allocate: already allocated")
        if self.linear_hidden > 0:
            check(
                LIB.rmsnorm_tp_create_linear(self.rank, self.tp_size, self.num_max_rows,
                                             self.linear_hidden, self.device,
                                             ctypes.byref(self._comm)),
                "rmsnorm_tp_create_linear",
            )
            return
        check(
            LIB.rmsnorm_tp_create(self.rank, self.tp_size, self.num_max_rows, self.device,
                                  ctypes.byref(self._comm)),
            "rmsnorm_tp_create",
        )

    def get_ipc_handle(self) -> IpcHandle:
        buf = ctypes.create_string_buffer(_lib.HANDLE_BYTES)
        n = ctypes.c_size_t()
        check(LIB.rmsnorm_tp_export_handle(self._comm, buf, _lib.HANDLE_BYTES, ctypes.byref(n)),
              "rmsnorm_tp_export_handle")
        return IpcHandle(buf.raw[: n.value])

    def open_remote_handle(self, remote_rank: int, handle: IpcHandle) -> None:
        data = handle.to_bytes()
        check(LIB.rmsnorm_tp_open_peer(self._comm, remote_rank, data, len(data)),
              "rmsnorm_tp_open_peer")

    def attach_peer(self, remote_rank: int, mailbox_ptr: int) -> None:
        """Use an already-mapped device pointer as a peer's mailbox."""
        check(LIB.rmsnorm_tp_attach_peer(self._comm, remote_rank, ctypes.c_void_p(mailbox_ptr)),
              "rmsnorm_tp_attach_peer")

    def mailbox(self):
        """(device pointer, bytes) of this rank's mailbox."""
        p = ctypes.c_void_p()
        n = ctypes.c_size_t()
        check(LIB.rmsnorm_tp_mailbox(self._comm, ctypes.byref(p), ctypes.byref(n)), "rmsnorm_tp_mailbox")
        return p.value, n.value

    def finalize_setup(self) -> None:
        check(LIB.rmsnorm_tp_finalize(self._comm), "rmsnorm_tp_finalize")

    def destroy(self) -> None:
        if self._comm.value:
            comm, self._comm = self._comm, ctypes.c_void_p()
            check(LIB.rmsnorm_tp_destroy(comm), "rmsnorm_tp_destroy")

    # -- generation (reference __init__.py:31-37)
    def next_generation(self) -> int:
        self._generation += 1
        return self._generation

    @property
    def generation(self) -> int:
        return self._generation

    def launch(self, out: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, hidden: int,
               eps: float, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One forward launch on the current stream, without the module around it
        (the counterpart of the reference's launch_fused_rmsnorm binding,
        csrc/bindings.cpp:182-196, minus its generation argument). ``residual``:
        fused residual add, as in ``FusedTPRMSNorm.forward``."""
        _check_operands(x, weight)
        rows, hl = x.shape
        if residual is not None:
            _check_like("residual", residual, x)
            check(
                LIB.rmsnorm_tp_forward_residual(self._comm, out.data_ptr(), residual.data_ptr(),
                                                x.data_ptr(), weight.data_ptr(), rows, hl, hidden,
                                                _DTYPES[x.dtype], float(eps),
                                                _stream_of(x.device.index)),
                "rmsnorm_tp_forward_residual",
            )
            self.next_generation()
            return out
        check(
            LIB.rmsnorm_tp_forward(self._comm, out.data_ptr(), x.data_ptr(), weight.data_ptr(), rows,
                                   hl, hidden, _DTYPES[x.dtype], float(eps),
                                   _stream_of(x.device.index)),
            "rmsnorm_tp_forward",
        )
        self.next_generation()
        return out

    def launch_backward(self, dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, hidden: int,
                        eps: float):
        """One backward launch on the current stream (two generations); returns (dx, dw)."""
        dx, dw, ws, nbytes = _backward_operands(dy, x, weight)
        rows, hl = x.shape
        check(
            LIB.rmsnorm_tp_backward(self._comm, dx.data_ptr(), dw.data_ptr(), dy.data_ptr(),
                                    x.data_ptr(), weight.data_ptr(), rows, hl, hidden,
                                    _DTYPES[x.dtype], float(eps), ws.data_ptr(), nbytes,
                                    _stream_of(x.device.index)),
            "rmsnorm_tp_backward",
        )
        self.next_generation()
        self.next_generation()
        return dx, dw

    # -- failure detection / recovery
    def set_timeout(self, seconds: float) -> None:
        check(LIB.rmsnorm_tp_set_timeout(self._comm, int(seconds * 1e9)), "rmsnorm_tp_set_timeout")

    def set_profile(self, counters: Optional[torch.Tensor]) -> None:
        """Point later launches at 20 int64 device counters (see profile_counters), or None."""
        ptr = None if counters is None else ctypes.c_void_p(counters.data_ptr())
        check(LIB.rmsnorm_tp_set_profile(self._comm, ptr), "rmsnorm_tp_set_profile")

    def poll_error(self) -> int:
        code = ctypes.c_uint32()
        check(LIB.rmsnorm_tp_poll_error(self._comm, ctypes.byref(code)), "rmsnorm_tp_poll_error")
        return code.value

    def status(self) -> dict:
        info = _lib.StatusInfo()
        check(LIB.rmsnorm_tp_status(self._comm, ctypes.byref(info)), "rmsnorm_tp_status")
        return {name: getattr(info, name) for name, _ in info._fields_}

    def reset(self, generation: int = 0) -> None:
        check(LIB.rmsnorm_tp_reset(self._comm, generation), "rmsnorm_tp_reset")
        self._generation = generation

    def device_generation(self) -> int:
        g = ctypes.c_uint64()
        check(LIB.rmsnorm_tp_get_generation(self._comm, ctypes.byref(g)), "rmsnorm_tp_get_generation")
        return g.value

    @property
    def handle(self) -> int:
        return self._comm.value or 0


def exchange_handles(group, local_device: int, handle: IpcHandle):
    """Bootstrap exchange: every rank's (device id, mailbox handle), in rank order.

    One all_gather_object of (device, 128 handle bytes) per rank replaces the
    reference's two (device ids, then handle bytes; rmsnorm_tp/__init__.py:58-61,
    :71-76). Raises if a handle has the wrong size.
    """
    tp = dist.get_world_size(group)
    gathered = [None] * tp
    dist.all_gather_object(gathered, (int(local_device), handle.to_bytes()), group=group)
    devices = [int(g[0]) for g in gathered]
    handles = [IpcHandle().from_bytes(g[1]) for g in gathered]
    return devices, handles


class FusedTPRMSNorm:
    """Fused tensor-parallel RMSNorm over NVLink (reference rmsnorm_tp/__init__.py:40-135).

    ``FusedTPRMSNorm(hidden_dim, eps=1e-6, tp_group=None, num_max_rows=65536)``;
    ``forward(x, weight)`` with x ``[num_rows, local_hidden_dim]`` and weight
    ``[local_hidden_dim]`` (float32, bfloat16 or float16); ``destroy()``.
    Like the reference, the normalising width is ``local_hidden_dim * tp_size``
    (reference __init__.py:101) and ``hidden_dim`` is informational.
    ``forward`` is a collective: all ranks call it in the same order with the
    same number of rows.
    """

    def __init__(self, hidden_dim: int, eps: float = 1e-6, tp_group=None,
                 num_max_rows: int = 65536, timeout_s: Optional[float] = None):
        self.hidden_dim = hidden_dim
        self.eps = eps
        self.tp_group = tp_group
        self.num_max_rows = int(num_max_rows)
        self.tp_size = dist.get_world_size(tp_group) if tp_group else 1
        self.rank = dist.get_rank(tp_group) if tp_group else 0
        self.comm_buf: Optional[TPCommBuffer] = None
        self.device_ids: List[int] = [torch.cuda.current_device()] if torch.cuda.is_available() else []
        if self.tp_size == 1:
            return

        local_device = torch.cuda.current_device()
        self.comm_buf = TPCommBuffer(self.rank, self.tp_size, self.num_max_rows, local_device)
        self.comm_buf.allocate()
        if timeout_s is not None:
            self.comm_buf.set_timeout(timeout_s)
        handle = self.comm_buf.get_ipc_handle()
        self.device_ids, handles = exchange_handles(tp_group, local_device, handle)
        for i in range(self.tp_size):
            if i != self.rank:
                self.comm_buf.open_remote_handle(i, handles[i])
        self.comm_buf.finalize_setup()
        dist.barrier(group=tp_group)

    def forward(self, x: torch.Tensor, weight: torch.Tensor,
                out: Optional[torch.Tensor] = None,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = x * rsqrt(sum over the group of x^2 / (local_hidden_dim * tp_size) + eps) * weight.

        ``out`` (optional, not in the reference) receives the result instead of a
        fresh tensor; it must be contiguous with x's shape, dtype and device.
        ``residual`` (optional, not in the reference): fused residual add in the
        same kernel -- ``z = x + residual`` (rounded to x's dtype) is written back
        into ``residual`` (the updated residual stream) and normalised instead of
        x; ``residual`` must be x-shaped and must not overlap ``out``.
        """
        _check_operands(x, weight)
        if out is not None:
            _check_like("out", out, x)
        if residual is not None:
            _check_like("residual", residual, x)
        num_rows, local_hidden_dim = x.shape
        if self.tp_size == 1:
            return local_rmsnorm(x, weight, self.eps, out, residual)
        if num_rows > self.num_max_rows:  # reference __init__.py:109
            raise AssertionError(f"num_rows {num_rows} > num_max_rows {self.num_max_rows}")
        if x.device.index != self.comm_buf.device:
            raise AssertionError(
                f"x is on cuda:{x.device.index}, the communicator on cuda:{self.comm_buf.device}"
            )
        output = torch.empty_like(x) if out is None else out
        if residual is not None:
            check(
                LIB.rmsnorm_tp_forward_residual(self.comm_buf._comm, output.data_ptr(),
                                                residual.data_ptr(), x.data_ptr(), weight.data_ptr(),
                                                num_rows, local_hidden_dim,
                                                local_hidden_dim * self.tp_size, _DTYPES[x.dtype],
                                                float(self.eps), _stream_of(x.device.index)),
                "rmsnorm_tp_forward_residual",
            )
        else:
            check(
                LIB.rmsnorm_tp_forward(self.comm_buf._comm, output.data_ptr(), x.data_ptr(),
                                       weight.data_ptr(), num_rows, local_hidden_dim,
                                       local_hidden_dim * self.tp_size, _DTYPES[x.dtype],
                                       float(self.eps), _stream_of(x.device.index)),
                "rmsnorm_tp_forward",
            )
        self.comm_buf.next_generation()   # the device advanced its own on the launch
        return output

    __call__ = forward

    def backward(self, dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor):
        """Gradients ``(dx, dw)`` of ``forward(x, weight)`` for the output gradient ``dy``
        (no reference counterpart). A collective like ``forward``; it uses two of the
        group's generations (one exchange of sum(x^2), one of sum(dy * w * x) per row).
        ``dw`` is this rank's slice of the weight gradient."""
        if self.tp_size == 1:
            return local_rmsnorm_backward(dy, x, weight, self.eps)
        num_rows, local_hidden_dim = x.shape
        if num_rows > self.num_max_rows:
            raise AssertionError(f"num_rows {num_rows} > num_max_rows {self.num_max_rows}")
        dx, dw, ws, nbytes = _backward_operands(dy, x, weight)
        check(
            LIB.rmsnorm_tp_backward(self.comm_buf._comm, dx.data_ptr(), dw.data_ptr(), dy.data_ptr(),
                                    x.data_ptr(), weight.data_ptr(), num_rows, local_hidden_dim,
                                    local_hidden_dim * self.tp_size, _DTYPES[x.dtype],
                                    float(self.eps), ws.data_ptr(), nbytes,
                                    _stream_of(x.device.index)),
            "rmsnorm_tp_backward",
        )
        self.comm_buf.next_generation()
        self.comm_buf.next_generation()
        return dx, dw

    def forward_with_grad(self, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        """``forward`` recorded for autograd: ``backward`` runs this module's
        backward kernel (a collective, so every rank must run the backward pass)."""
        return _TPRMSNormFunction.apply(self, x, weight)

    # -- failure detection / recovery (no reference counterpart)
    def status(self) -> dict:
        return self.comm_buf.status() if self.comm_buf else {"code": 0}

    def reset(self, generation: int = 0) -> None:
        """Collective recovery after a device failure: wait, zero the mailbox,
        set the generation, between two group barriers."""
        if self.comm_buf is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.tp_group)
        self.comm_buf.reset(generation)
        dist.barrier(group=self.tp_group)

    def destroy(self) -> None:
        """Free the mailbox. Unlike the reference (csrc/bindings.cpp:84-99) the
        ranks first wait for each other, so no peer can still be writing into it."""
        if self.comm_buf is not None:
            torch.cuda.synchronize()
            if dist.is_available() and dist.is_initialized():
                dist.barrier(group=self.tp_group)
            self.comm_buf.destroy()
            self.comm_buf = None


def _check_linear_operands(a: torch.Tensor, linear_weight: torch.Tensor,
                           norm_weight: torch.Tensor, hidden: int, tp: int) -> None:
    for name, t in (("a", a), ("linear_weight", linear_weight), ("norm_weight", norm_weight)):
        if not t.is_contiguous():
            raise AssertionError(f"{name} must be contiguous")
        if not t.is_cuda or t.device != a.device:
            raise AssertionError(f"{name} must be a CUDA tensor on a's device")
        if t.dtype != a.dtype:
            raise AssertionError(f"{name} must have a's dtype ({a.dtype}), got {t.dtype}")
    if a.dtype not in (torch.bfloat16, torch.float16):
        raise AssertionError(f"the tensor-core path takes bfloat16 or float16, got {a.dtype}")
    if a.dim() != 2 or linear_weight.dim() != 2 or linear_weight.shape != (hidden, a.shape[1]):
        raise AssertionError(
            f"a must be [rows, k_local] and linear_weight [hidden={hidden}, k_local], got "
            f"{tuple(a.shape)} and {tuple(linear_weight.shape)}")
    if norm_weight.shape != (hidden // tp,):
        raise AssertionError(f"norm_weight must be [{hidden // tp}], got {tuple(norm_weight.shape)}")


class FusedTPLinearRMSNorm:
    """Row-parallel linear -> reduce-scatter -> (residual add) -> TP RMSNorm, one
    kernel per call (no reference counterpart: the reference normalises the
    output of an NCCL reduction with its AllReduce path, bench_rmsnorm_tp.py:16-22).

    ``FusedTPLinearRMSNorm(hidden_dim, eps=1e-6, tp_group=None, num_max_rows=4096)``;
    ``forward(a, linear_weight, norm_weight, residual=None, out=None)`` with ``a``
    ``[rows, k_local]`` (this rank's slice of the linear's input features),
    ``linear_weight`` ``[hidden_dim, k_local]`` (nn.Linear layout), ``norm_weight``
    ``[hidden_dim / tp]``; returns this rank's ``[rows, hidden_dim / tp]`` columns of
    ``rmsnorm(sum over ranks of a_r @ linear_weight_r^T (+ residual))``. ``residual``
    (``[rows, hidden_dim / tp]``) is updated in place with the sum. bf16 or fp16;
    k_local a multiple of 64, hidden_dim a multiple of 128 * tp. A collective:
    every rank calls it in the same order with the same number of rows.
    """

    def __init__(self, hidden_dim: int, eps: float = 1e-6, tp_group=None,
                 num_max_rows: int = 4096, timeout_s: Optional[float] = None):
        self.hidden_dim = int(hidden_dim)
        self.eps = eps
        self.tp_group = tp_group
        self.num_max_rows = int(num_max_rows)
        self.tp_size = dist.get_world_size(tp_group) if tp_group else 1
        self.rank = dist.get_rank(tp_group) if tp_group else 0
        local_device = torch.cuda.current_device()
        self.comm_buf = TPCommBuffer(self.rank, self.tp_size, self.num_max_rows, local_device,
                                     linear_hidden=self.hidden_dim)
        self.comm_buf.allocate()
        if timeout_s is not None:
            self.comm_buf.set_timeout(timeout_s)
        if self.tp_size > 1:
            handle = self.comm_buf.get_ipc_handle()
            _, handles = exchange_handles(tp_group, local_device, handle)
            for i in range(self.tp_size):
                if i != self.rank:
                    self.comm_buf.open_remote_handle(i, handles[i])
        self.comm_buf.finalize_setup()
        if self.tp_size > 1:
            dist.barrier(group=tp_group)

    def forward(self, a: torch.Tensor, linear_weight: torch.Tensor, norm_weight: torch.Tensor,
                residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        _check_linear_operands(a, linear_weight, norm_weight, self.hidden_dim, self.tp_size)
        rows = a.shape[0]
        if rows > self.num_max_rows:
            raise AssertionError(f"num_rows {rows} > num_max_rows {self.num_max_rows}")
        hl = self.hidden_dim // self.tp_size
        if out is None:
            out = torch.empty(rows, hl, dtype=a.dtype, device=a.device)
        elif out.shape != (rows, hl) or out.dtype != a.dtype or not out.is_contiguous():
            raise AssertionError(f"out must be contiguous [{rows}, {hl}] of a's dtype")
        if residual is not None and (residual.shape != (rows, hl) or residual.dtype != a.dtype
                                     or not residual.is_contiguous()):
            raise AssertionError(f"residual must be contiguous [{rows}, {hl}] of a's dtype")
        check(
            LIB.rmsnorm_tp_linear_forward(self.comm_buf._comm, out.data_ptr(),
                                          None if residual is None else residual.data_ptr(),
                                          a.data_ptr(), linear_weight.data_ptr(),
                                          norm_weight.data_ptr(), rows, a.shape[1],
                                          _DTYPES[a.dtype], float(self.eps),
                                          _stream_of(a.device.index)),
            "rmsnorm_tp_linear_forward",
        )
        self.comm_buf.next_generation()
        return out

    __call__ = forward

    def status(self) -> dict:
        return self.comm_buf.status()

    def destroy(self) -> None:
        if self.comm_buf is not None:
            torch.cuda.synchronize()
            if self.tp_size > 1 and dist.is_available() and dist.is_initialized():
                dist.barrier(group=self.tp_group)
            self.comm_buf.destroy()
            self.comm_buf = None


class EmulatedTPLinearGroup:
    """Every rank of a FusedTPLinearRMSNorm group on ONE GPU (one cooperative
    launch, rank = blockIdx.y), for tests without several GPUs."""

    def __init__(self, tp_size: int, hidden_dim: int, eps: float = 1e-6,
                 num_max_rows: int = 4096, device: Optional[int] = None,
                 timeout_s: Optional[float] = None):
        if not 2 <= tp_size <= _lib.MAX_TP:
            raise ValueError(f"tp_size {tp_size} outside [2, {_lib.MAX_TP}]")
        self.tp_size, self.hidden_dim, self.eps = tp_size, int(hidden_dim), eps
        self.num_max_rows = int(num_max_rows)
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.bufs = [TPCommBuffer(r, tp_size, self.num_max_rows, self.device,
                                  linear_hidden=self.hidden_dim) for r in range(tp_size)]
        for b in self.bufs:
            b.allocate()
            if timeout_s is not None:
                b.set_timeout(timeout_s)
        boxes = [b.mailbox()[0] for b in self.bufs]
        for b in self.bufs:
            for q in range(tp_size):
                if q != b.rank:
                    b.attach_peer(q, boxes[q])
            b.finalize_setup()

    def forward(self, as_: Sequence[torch.Tensor], linear_weights: Sequence[torch.Tensor],
                norm_weights: Sequence[torch.Tensor],
                residuals: Optional[Sequence[torch.Tensor]] = None) -> List[torch.Tensor]:
        tp = self.tp_size
        for a, w, g in zip(as_, linear_weights, norm_weights):
            _check_linear_operands(a, w, g, self.hidden_dim, tp)
        rows, k = as_[0].shape
        hl = self.hidden_dim // tp
        outs = [torch.empty(rows, hl, dtype=as_[0].dtype, device=as_[0].device) for _ in range(tp)]
        P = ctypes.c_void_p * tp
        rptr = None if residuals is None else P(*[r.data_ptr() for r in residuals])
        check(
            LIB.rmsnorm_tp_linear_forward_emulated(
                P(*[b._comm.value for b in self.bufs]), tp, P(*[o.data_ptr() for o in outs]), rptr,
                P(*[a.data_ptr() for a in as_]), P(*[w.data_ptr() for w in linear_weights]),
                P(*[g.data_ptr() for g in norm_weights]), rows, k, _DTYPES[as_[0].dtype],
                float(self.eps), _stream_of(as_[0].device.index)),
            "rmsnorm_tp_linear_forward_emulated",
        )
        for b in self.bufs:
            b.next_generation()
        return outs

    def destroy(self) -> None:
        for b in self.bufs:
            b.destroy()


class EmulatedTPGroup:
    """All ranks of a TP group on ONE GPU, for testing the exchange without
    several GPUs: each rank gets its own mailbox and device state, the peers are
    attached to each other's (local) mailboxes, and ``forward`` runs every rank
    in one cooperative launch (rank = blockIdx.y), so no two kernels that wait
    on each other are ever launched separately on one GPU."""

    def __init__(self, tp_size: int, eps: float = 1e-6, num_max_rows: int = 65536,
                 device: Optional[int] = None, timeout_s: Optional[float] = None):
        if not 2 <= tp_size <= _lib.MAX_TP:
            raise ValueError(f"tp_size {tp_size} outside [2, {_lib.MAX_TP}]")
        self.tp_size = tp_size
        self.eps = eps
        self.num_max_rows = num_max_rows
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.bufs = [TPCommBuffer(r, tp_size, num_max_rows, self.device) for r in range(tp_size)]
        for b in self.bufs:
            b.allocate()
            if timeout_s is not None:
                b.set_timeout(timeout_s)
        boxes = [b.mailbox()[0] for b in self.bufs]
        for b in self.bufs:
            for q in range(tp_size):
                if q != b.rank:
                    b.attach_peer(q, boxes[q])
            b.finalize_setup()

    def forward(self, xs: Sequence[torch.Tensor], weights: Sequence[torch.Tensor],
                outs: Optional[Sequence[torch.Tensor]] = None,
                residuals: Optional[Sequence[torch.Tensor]] = None) -> List[torch.Tensor]:
        """Every rank's forward in one launch; ``residuals`` (one per rank): the
        fused residual add of ``FusedTPRMSNorm.forward``."""
        tp = self.tp_size
        if len(xs) != tp or len(weights) != tp:
            raise AssertionError(f"need {tp} x slices and {tp} weights")
        for x, w in zip(xs, weights):
            _check_operands(x, w)
        rows, hl = xs[0].shape
        if any(tuple(x.shape) != (rows, hl) for x in xs) or any(x.dtype != xs[0].dtype for x in xs):
            raise AssertionError("every rank needs the same shape and dtype")
        if rows > self.num_max_rows:
            raise AssertionError(f"num_rows {rows} > num_max_rows {self.num_max_rows}")
        if outs is None:
            outs = [torch.empty_like(x) for x in xs]
        P = ctypes.c_void_p * tp
        comms = P(*[b._comm.value for b in self.bufs])
        optr = P(*[o.data_ptr() for o in outs])
        xptr = P(*[x.data_ptr() for x in xs])
        wptr = P(*[w.data_ptr() for w in weights])
        if residuals is not None:
            if len(residuals) != tp:
                raise AssertionError(f"need {tp} residuals")
            for r, x in zip(residuals, xs):
                _check_like("residual", r, x)
            rptr = P(*[r.data_ptr() for r in residuals])
            check(
                LIB.rmsnorm_tp_forward_emulated_residual(comms, tp, optr, rptr, xptr, wptr, rows, hl,
                                                         _DTYPES[xs[0].dtype], float(self.eps),
                                                         _stream_of(xs[0].device.index)),
                "rmsnorm_tp_forward_emulated_residual",
            )
            for b in self.bufs:
                b.next_generation()
            return list(outs)
        check(
            LIB.rmsnorm_tp_forward_emulated(comms, tp, optr, xptr, wptr, rows, hl,
                                            _DTYPES[xs[0].dtype], float(self.eps),
                                            _stream_of(xs[0].device.index)),
            "rmsnorm_tp_forward_emulated",
        )
        for b in self.bufs:
            b.next_generation()
        return list(outs)

    def backward(self, dys: Sequence[torch.Tensor], xs: Sequence[torch.Tensor],
                 weights: Sequence[torch.Tensor]):
        """Every rank's backward in one launch; returns (dxs, dws)."""
        tp = self.tp_size
        if len(xs) != tp or len(weights) != tp or len(dys) != tp:
            raise AssertionError(f"need {tp} dy, x and weight slices")
        ops = [_backward_operands(dy, x, w) for dy, x, w in zip(dys, xs, weights)]
        rows, hl = xs[0].shape
        if any(tuple(x.shape) != (rows, hl) for x in xs) or any(x.dtype != xs[0].dtype for x in xs):
            raise AssertionError("every rank needs the same shape and dtype")
        P = ctypes.c_void_p * tp
        comms = P(*[b._comm.value for b in self.bufs])
        check(
            LIB.rmsnorm_tp_backward_emulated(
                comms, tp, P(*[o[0].data_ptr() for o in ops]), P(*[o[1].data_ptr() for o in ops]),
                P(*[d.data_ptr() for d in dys]), P(*[x.data_ptr() for x in xs]),
                P(*[w.data_ptr() for w in weights]), rows, hl, _DTYPES[xs[0].dtype],
                float(self.eps), P(*[o[2].data_ptr() for o in ops]), ops[0][3],
                _stream_of(xs[0].device.index)),
            "rmsnorm_tp_backward_emulated",
        )
        for b in self.bufs:
            b.next_generation()
            b.next_generation()
        return [o[0] for o in ops], [o[1] for o in ops]

    def reset(self, generation: int = 0) -> None:
        for b in self.bufs:
            b.reset(generation)

    def destroy(self) -> None:
        for b in self.bufs:
            b.destroy()


class _TPRMSNormFunction(torch.autograd.Function):
    """Autograd around FusedTPRMSNorm: forward kernel, backward kernel."""

    @staticmethod
    def forward(ctx, module, x, weight):
        ctx.module = module
        ctx.save_for_backward(x, weight)
        return module.forward(x, weight)

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        dx, dw = ctx.module.backward(dy.contiguous(), x, weight)
        return None, dx, dw


PROFILE_COUNTERS = 20


def profile_counters(device=None) -> torch.Tensor:
    """Fresh in-kernel counters for TPCommBuffer.set_profile: int64[20] =
    [wait ns, slow waits, fast waits, earliest CTA start, latest CTA end,
    sum of CTA start -> partials pushed, sum of pushed -> CTA end, CTAs with the
    pushed mark, sum of CTA start -> end, CTAs, sum of launch spans, launches,
    sum of gaps between launches, gaps, 3 x scratch, sum of CTA start delays
    after the previous launch's end, CTAs counted there, unused] (ns of the
    GPU timer)."""
    t = torch.zeros(PROFILE_COUNTERS, dtype=torch.int64, device=device or "cuda")
    t[3] = -1    # UINT64_MAX for the atomicMin of the start time
    t[14] = -1   # and for the per-launch first start
    return t


def profile_summary(v) -> dict:
    """Readable means of profile_counters values (a list of 20 ints)."""
    u = [x & 0xFFFFFFFFFFFFFFFF for x in v]
    polls = u[1] + u[2]
    d = lambda a, b: round(u[a] / u[b] / 1e3, 3) if u[b] else None
    return {"polls": polls, "slow_poll_share": round(u[1] / max(1, polls), 4),
            "mean_wait_us": round(u[0] / max(1, u[1]) / 1e3, 3),
            "launch_span_us": d(10, 11), "launch_gap_us": d(12, 13),
            "cta_start_delay_us": d(17, 18),
            "cta_us": d(8, 9), "cta_load_reduce_push_us": d(5, 7),
            "cta_poll_store_us": d(6, 7)}


def plan(rows: int, local_hidden: int, dtype: torch.dtype, aligned: bool = True, tp: int = 1,
         resident_ctas: int = 148 * 2) -> dict:
    """Launch plan the forward call would use (host arithmetic only)."""
    info = _lib.PlanInfo()
    check(LIB.rmsnorm_tp_plan(rows, local_hidden, dtype_code(dtype), int(aligned), tp,
                              resident_ctas, ctypes.byref(info)), "rmsnorm_tp_plan")
    return {name: getattr(info, name) for name, _ in info._fields_}


def plan_coverage(plan_dict: dict, rows: int):
    """Per-row visit counts of the row -> team mapping (host replica of the kernels' walk)."""
    info = _lib.PlanInfo(**{k: plan_dict[k] for k, _ in _lib.PlanInfo._fields_})
    counts = (ctypes.c_int32 * max(rows, 1))()
    check(LIB.rmsnorm_tp_plan_coverage(ctypes.byref(info), rows, counts), "rmsnorm_tp_plan_coverage")
    return list(counts)[:rows]


_FAMILIES = {"auto": _lib.FAMILY_AUTO, "register": _lib.FAMILY_REGISTER, "bulk": _lib.FAMILY_BULK,
             "batch": _lib.FAMILY_BATCH}


def set_kernel_family(family: str) -> None:
    """Process-wide kernel family: "auto", "register", "bulk" or "batch" (tests, benchmarks)."""
    check(LIB.rmsnorm_tp_set_kernel_family(_FAMILIES[family]), "rmsnorm_tp_set_kernel_family")


def get_kernel_family() -> str:
    return {v: k for k, v in _FAMILIES.items()}[LIB.rmsnorm_tp_get_kernel_family()]


_PUSH_MODES = {"packed": _lib.PUSH_PACKED, "release": _lib.PUSH_RELEASE}


def set_push_mode(mode: str) -> None:
    """Process-wide exchange encoding: "packed" (one 64-bit {tag, partial} store, the
    default) or "release" (the partial, then a release-stored tag: the reference's
    scheme, for comparison). Every rank of a group must use the same one."""
    check(LIB.rmsnorm_tp_set_push_mode(_PUSH_MODES[mode]), "rmsnorm_tp_set_push_mode")


def get_push_mode() -> str:
    return {v: k for k, v in _PUSH_MODES.items()}[LIB.rmsnorm_tp_get_push_mode()]


def set_dependent_launch(enable: bool) -> None:
    """Process-wide programmatic dependent launch of forward kernels (default on)."""
    check(LIB.rmsnorm_tp_set_dependent_launch(1 if enable else 0), "rmsnorm_tp_set_dependent_launch")


def get_dependent_launch() -> bool:
    return LIB.rmsnorm_tp_get_dependent_launch() == 1


def tag_of(generation: int) -> int:
    return LIB.rmsnorm_tp_tag_of(generation)


def buffer_of(generation: int) -> int:
    return LIB.rmsnorm_tp_buffer_of(generation)
