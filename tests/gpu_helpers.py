"""Helpers shared by the GPU tests: torch <-> oracle arrays, raw device views."""
import numpy as np
import torch

from oracle import tp_rmsnorm as O

TORCH_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
NAMES = {v: k for k, v in TORCH_DTYPES.items()}


def to_np(t: torch.Tensor) -> np.ndarray:
    """Tensor -> oracle storage (f32 float32, bf16 uint16 bits, f16 float16)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def from_np(dtype: str, a: np.ndarray, device="cuda") -> torch.Tensor:
    if dtype == "bf16":
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(a).copy())
    return t.to(device)


def out_f32(dtype: str, t: torch.Tensor) -> np.ndarray:
    return O.to_f32(dtype, to_np(t))


def check_against_oracle(dtype, xs, ws, eps, outs, reference=True):
    """Compare kernel outputs (tensors in x's dtype) with the oracle in x's dtype.

    reference=True: the reference's AllReduce path (the parity bar);
    reference=False: the fused formula (fp32 squares), e.g. where fp16 squares overflow.
    """
    xn = [to_np(x) for x in xs]
    wn = [to_np(w) for w in ws]
    want = (O.allreduce_path if reference else O.fused_path)(xn, wn, eps, dtype)
    results = []
    for got, ref in zip(outs, want):
        r = O.compare(dtype, out_f32(dtype, got), O.round_to(dtype, ref))
        results.append(r)
    return results


class RawDeviceArray:
    """A typed view of raw device memory (e.g. a mailbox), usable by torch.as_tensor."""

    def __init__(self, ptr: int, nbytes: int, typestr: str = "<i8", itemsize: int = 8):
        self.__cuda_array_interface__ = {
            "shape": (nbytes // itemsize,),
            "typestr": typestr,
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }


def device_view(ptr: int, nbytes: int) -> torch.Tensor:
    return torch.as_tensor(RawDeviceArray(ptr, nbytes), device="cuda")


def slot_index(buf, src, tp, nmax, row):
    return (buf * tp + src) * nmax + row


def pack_slots(partials: np.ndarray, tag: int) -> np.ndarray:
    """{fp32 partial, tag} mailbox words as int64."""
    lo = np.asarray(partials, dtype=np.float32).view(np.uint32).astype(np.uint64)
    w = (np.uint64(tag) << np.uint64(32)) | lo
    return w.view(np.int64)
