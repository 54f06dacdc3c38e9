"""Host side of the row kernels (softmax, log-softmax, mean, L2 norm, and
the fused LayerNorm / RMSNorm).

Reductions run on a contiguous ``[outer, n, inner]`` view.  A single reduced
dimension keeps the tensor's layout (column mode when it is not the last
dimension); several reduced dimensions are first moved to the end with one
copy so that each output owns one contiguous row of length ``n``.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib, tracing


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
    with tracing.span("softmax", f"bio_softmax [rows={outer * inner}, n={n}, log={int(log)}]", 0,
                  xin.numel() * (xin.element_size() + out.element_size()), xin.element_size()):
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
    with tracing.span(kind, f"bio_reduce [{kind}, outputs={outer * inner}, n={n}]", 0,
                  xin.numel() * xin.element_size() + out.numel() * out.element_size(),
                  xin.element_size()):
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


def norm(
    x: torch.Tensor,
    normalized_shape,
    weight: torch.Tensor | None,
    bias: torch.Tensor | None,
    eps: float,
    rms: bool,
    want_stats: bool = False,
):
    """Fused LayerNorm (rms=False) / RMSNorm (rms=True) over the trailing
    ``normalized_shape`` dims through ``bio_norm``.  Returns the output, plus
    (mean, rstd) in fp32 with the statistics shape of aten::native_layer_norm
    (leading dims, then ones) when ``want_stats``."""
    _check_float(x)
    shape = tuple(int(s) for s in normalized_shape)
    nd = len(shape)
    if nd == 0 or tuple(x.shape[x.ndim - nd:]) != shape or x.ndim < nd:
        raise RuntimeError(
            f"normalized_shape {list(shape)} does not match the trailing dims of input "
            f"{list(x.shape)}")
    n = math.prod(shape)
    xin = x.contiguous()
    rows = xin.numel() // n if n > 0 else 0
    out = torch.empty_like(xin)
    stat_shape = tuple(x.shape[: x.ndim - nd]) + (1,) * nd
    mean = rstd = None
    if want_stats:
        mean = torch.empty(stat_shape, dtype=torch.float32, device=x.device)
        rstd = torch.empty(stat_shape, dtype=torch.float32, device=x.device)
    if out.numel() == 0:
        if want_stats and n == 0:
            mean.zero_()
            rstd.fill_(float("inf"))
        return (out, mean, rstd) if want_stats else out
    w_dtype = None
    if weight is not None:
        if weight.numel() != n:
            raise RuntimeError("weight must have normalized_shape elements")
        weight = weight.contiguous()
        w_dtype = weight.dtype
    if bias is not None:
        if bias.numel() != n:
            raise RuntimeError("bias must have normalized_shape elements")
        bias = bias.to(w_dtype or bias.dtype).contiguous()
        w_dtype = w_dtype or bias.dtype
    w_dtype = w_dtype or x.dtype
    if w_dtype not in _lib.DTYPE_CODE:
        raise RuntimeError(f"unsupported weight dtype: {w_dtype}")
    with tracing.span("norm", f"bio_norm [{'rms' if rms else 'layer'}, rows={rows}, n={n}]", 0,
                      2 * xin.numel() * xin.element_size(), xin.element_size()):
        _lib.check(
            _lib.load().bio_norm(
                _lib.BIO_NORM_RMS if rms else _lib.BIO_NORM_LAYER,
                _lib.DTYPE_CODE[xin.dtype],
                _lib.DTYPE_CODE[w_dtype],
                ctypes.c_void_p(xin.data_ptr()),
                ctypes.c_void_p(weight.data_ptr() if weight is not None else 0),
                ctypes.c_void_p(bias.data_ptr() if bias is not None else 0),
                ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(mean.data_ptr() if mean is not None else 0),
                ctypes.c_void_p(rstd.data_ptr() if rstd is not None else 0),
                rows,
                n,
                n,
                n,
                float(eps),
                x.device.index,
                _lib.stream_of(x),
            ),
            "bio_norm",
        )
    return (out, mean, rstd) if want_stats else out
