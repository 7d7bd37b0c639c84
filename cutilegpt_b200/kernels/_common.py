"""Input handling shared by the reference-named operators."""
from __future__ import annotations

import torch


def as_cuda(x, name: str = "tensor") -> torch.Tensor:
    """Accepts a CUDA torch tensor, or any DLPack producer (e.g. a CuPy array).

    Mirrors the reference's input rule (device arrays only; anything else is
    a ValueError, e.g. cutile_gpt/kernels/linear.py:125-126).
    """
    if isinstance(x, torch.Tensor):
        t = x
    elif hasattr(x, "__dlpack__"):
        t = torch.from_dlpack(x)
    else:
        raise ValueError(f"{name}: expected a CUDA tensor, got {type(x).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name}: tensors must be on a CUDA device")
    return t


def same_dtype(ref: torch.Tensor, *others: torch.Tensor) -> None:
    for o in others:
        if o is not None and o.dtype != ref.dtype:
            raise ValueError(f"dtype mismatch: {ref.dtype} vs {o.dtype}")
