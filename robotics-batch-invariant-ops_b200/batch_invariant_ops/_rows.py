"""Host side of the row kernels (softmax, log-softmax, mean, L2 norm).

Reductions run on a contiguous ``[outer, n, inner]`` view.  A single reduced
dimension keeps the tensor's layout (column mode when it is not the last
dimension); several reduced dimensions are first moved to the end with one
copy so that each output owns one contiguous row of length ``n``.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib


def _check_float(t: torch.Tensor) -> None:
    if t.dtype not in _lib.DTYPE_CODE:
        raise AssertionError(f"unsupported dtype: {t.dtype}")


def softmax(x: torch.Tensor, dim: int, dtype: torch.dtype | None, log: bool) -> torch.Tensor:
    _check_float(x)
    out_dtype = dtype or x.dtype
    if out_dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"unsupported softmax output dtype: {out_dtype}")
    if x.ndim == 0:
        xin = x.reshape(1)
        dim = 0
    else:
        xin = x
        dim %= x.ndim
    xin = xin.contiguous()
    shape = xin.shape
    outer = math.prod(shape[:dim])
    n = shape[dim]
    inner = math.prod(shape[dim + 1 :])
    out = torch.empty(shape, dtype=out_dtype, device=x.device)
    if out.numel() == 0:
        return out.reshape(x.shape)
    _lib.check(
        _lib.load().bio_softmax(
            _lib.DTYPE_CODE[xin.dtype],
            _lib.DTYPE_CODE[out_dtype],
            ctypes.c_void_p(xin.data_ptr()),
            ctypes.c_void_p(out.data_ptr()),
            outer,
            n,
            inner,
            1 if log else 0,
            x.device.index,
            _lib.stream_of(x),
        ),
        "bio_softmax",
    )
    return out.reshape(x.shape)


def reduce_dims(
    x: torch.Tensor,
    dims: tuple[int, ...],
    keepdim: bool,
    *,
    kind: str,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Mean (``kind="mean"``) or Euclidean norm (``kind="l2norm"``) over ``dims``."""
    _check_float(x)
    out_dtype = out_dtype or x.dtype
    ndim = x.ndim
    dims = tuple(sorted(d % ndim for d in dims)) if ndim else ()
    kept = tuple(d for d in range(ndim) if d not in dims)
    out_shape = tuple(1 if d in dims else x.shape[d] for d in range(ndim)) if keepdim else tuple(
        x.shape[d] for d in kept
    )
    if len(dims) <= 1:
        xin = x.contiguous()
        if dims:
            d = dims[0]
            outer = math.prod(x.shape[:d])
            n = x.shape[d]
            inner = math.prod(x.shape[d + 1 :])
        else:
            outer, n, inner = max(x.numel(), 1), 1, 1
    else:
        xin = x.permute(*kept, *dims).contiguous()
        outer = math.prod(x.shape[d] for d in kept)
        n = math.prod(x.shape[d] for d in dims)
        inner = 1
    out = torch.empty(out_shape, dtype=out_dtype, device=x.device)
    if out.numel() == 0:
        return out
    code = {"mean": 0, "l2norm": 1}[kind]
    _lib.check(
        _lib.load().bio_reduce(
            code,
            _lib.DTYPE_CODE[xin.dtype],
            _lib.DTYPE_CODE[out_dtype],
            ctypes.c_void_p(xin.data_ptr()),
            ctypes.c_void_p(out.data_ptr()),
            outer,
            n,
            inner,
            x.device.index,
            _lib.stream_of(x),
        ),
        "bio_reduce",
    )
    return out
