"""Host side of the convolution family.

Regular convolution (1-D, 2-D, 3-D, any groups/stride/padding/dilation):
``bio_im2col`` builds patches[B, G, L, Kpad]; then ONE bio_gemm launch runs an
independent fixed-schedule GEMM per (sample, group):
out[b, g*Og:(g+1)*Og, L] = W_g[Og, K] @ patches[b, g]^T, bias added per output
channel in the GEMM epilogue.  The output lands directly in NC[D][H]W layout.
Depthwise 1-D convolution uses a direct kernel.

Transposed convolution with stride == kernel (padding 0, dilation 1), the
reference's orientation (batch_invariant_ops.py:835-861): per (sample,
group) C[P, Og*kvol] = X[b, g]^T @ W_g, and for 16-bit types one
``bio_conv_transpose`` GEMM whose epilogue rounds, adds the bias and writes
each kernel row straight into the output layout.  fp32 (and shapes whose
sizes break the tensor-map alignment) run the GEMM into a buffer and then
``bio_conv_transpose_scatter``.

Assertion messages follow the reference (batch_invariant_ops.py:497-941).
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _gemm, _lib, tracing


class _Geom(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("channels", ctypes.c_int64),
        ("groups", ctypes.c_int64),
        ("inp", ctypes.c_int64 * 3),
        ("kernel", ctypes.c_int64 * 3),
        ("stride", ctypes.c_int64 * 3),
        ("padding", ctypes.c_int64 * 3),
        ("dilation", ctypes.c_int64 * 3),
        ("out", ctypes.c_int64 * 3),
    ]


def _expand(values, nd: int, name: str) -> tuple[int, ...]:
    values = tuple(values)
    if len(values) == 1:
        return values * nd
    if nd == 1:
        assert len(values) == 1, f"{name} must have one value, got {values!r}"
    elif nd == 2:
        assert len(values) == 2, f"{name} must have one or two values, got {values!r}"
    else:
        assert len(values) == 3, f"{name} must have one or three values, got {values!r}"
    return tuple(int(v) for v in values)


def _pad3(t: tuple[int, ...], fill: int) -> tuple[int, int, int]:
    return (fill,) * (3 - len(t)) + tuple(t)


def _geom(batch, channels, groups, inp, kernel, stride, padding, dilation, out) -> _Geom:
    g = _Geom()
    g.batch, g.channels, g.groups = batch, channels, groups
    for field, vals, fill in (
        ("inp", inp, 1),
        ("kernel", kernel, 1),
        ("stride", stride, 1),
        ("padding", padding, 0),
        ("dilation", dilation, 1),
        ("out", out, 1),
    ):
        arr = getattr(g, field)
        for i, v in enumerate(_pad3(vals, fill)):
            arr[i] = v
    return g


def conv_nd(input, weight, bias, stride, padding, dilation, transposed, output_padding, groups, nd):
    names = {1: "only 1-D convolution is supported", 2: "only 2-D convolution is supported",
             3: "only 3-D convolution is supported"}
    assert input.ndim == nd + 2 and weight.ndim == nd + 2, names[nd]
    assert not transposed, "transposed convolution is not supported"
    assert all(
        value == 0 for value in output_padding
    ), f"output_padding requires transposed convolution, got {output_padding!r}"
    assert input.dtype == weight.dtype and (
        bias is None or bias.dtype == input.dtype
    ), "Incompatible dtypes"
    assert input.shape[1] == weight.shape[1] * groups, "Incompatible channel dimensions"
    assert weight.shape[0] % groups == 0, "output channels must be divisible by groups"
    assert input.dtype in _lib.DTYPE_CODE, f"unsupported dtype: {input.dtype}"
    if not input.is_cuda:
        raise AssertionError("batch-invariant operators require CUDA tensors")

    stride = _expand(stride, nd, "stride")
    padding = _expand(padding, nd, "padding")
    dilation = _expand(dilation, nd, "dilation")
    ksize = tuple(weight.shape[2:])
    out_shape = tuple(
        (input.shape[2 + i] + 2 * padding[i] - dilation[i] * (ksize[i] - 1) - 1) // stride[i] + 1
        for i in range(nd)
    )
    batch, channels = input.shape[:2]
    cout = weight.shape[0]
    out = torch.empty((batch, cout, *out_shape), device=input.device, dtype=input.dtype)
    if batch == 0 or out.numel() == 0:
        return out
    lib = _lib.load()
    stream = _lib.stream_of(input)
    dev = input.device.index
    dtype_code = _lib.DTYPE_CODE[input.dtype]
    x = input.contiguous()
    bias_c = bias.contiguous() if bias is not None else None

    if nd == 1 and groups == channels == cout and weight.shape[1] == 1:
        w = weight.contiguous()
        with tracing.span("conv", f"bio_depthwise_conv1d [B={batch}, C={channels}, L={out_shape[0]}, k={ksize[0]}]",
                      2.0 * out.numel() * ksize[0],
                      (x.numel() + out.numel()) * x.element_size(), x.element_size()):
            _lib.check(
                lib.bio_depthwise_conv1d(
                    dtype_code,
                    ctypes.c_void_p(x.data_ptr()),
                    ctypes.c_void_p(w.data_ptr()),
                    ctypes.c_void_p(bias_c.data_ptr() if bias_c is not None else 0),
                    ctypes.c_void_p(out.data_ptr()),
                    batch,
                    channels,
                    input.shape[-1],
                    out_shape[0],
                    ksize[0],
                    stride[0],
                    padding[0],
                    dilation[0],
                    dev,
                    stream,
                ),
                "bio_depthwise_conv1d",
            )
        return out

    cg = channels // groups
    og = cout // groups
    kvol = math.prod(ksize)
    k = cg * kvol
    kpad = (k + 7) // 8 * 8
    lvol = math.prod(out_shape)
    patches = torch.empty((batch, groups, lvol, kpad), device=input.device, dtype=input.dtype)
    geom = _geom(batch, channels, groups, input.shape[2:], ksize, stride, padding, dilation,
                 out_shape)
    with tracing.span("conv", f"bio_im2col [B={batch}, G={groups}, L={lvol}, K={k}]", 0,
                  (x.numel() + patches.numel()) * x.element_size(), x.element_size()):
        _lib.check(
            lib.bio_im2col(
                dtype_code,
                ctypes.c_void_p(x.data_ptr()),
                ctypes.byref(geom),
                ctypes.c_void_p(patches.data_ptr()),
                kpad,
                dev,
                stream,
            ),
            "bio_im2col",
        )
    w = weight.contiguous()
    opa = _gemm.operand_a(w, batch, groups, og, k, k, 1, 0, og * k)
    opb = _gemm.Operand(patches, patches.data_ptr(), 1, kpad, groups * lvol * kpad, lvol * kpad)
    _gemm.launch(
        opa,
        opb,
        out,
        batch1=batch,
        batch2=groups,
        m=og,
        n=lvol,
        k=k,
        c_sm=lvol,
        c_sn=1,
        c_s1=cout * lvol,
        c_s2=og * lvol,
        bias=bias_c,
        bias_per_row=True,
        bias_s2=og,
    )
    return out


def conv_transpose_nd(input, weight, bias, stride, padding, dilation, output_padding, groups, nd):
    names = {2: "only 2-D convolution is supported", 3: "only 3-D convolution is supported"}
    assert input.ndim == nd + 2 and weight.ndim == nd + 2, names[nd]
    assert input.dtype == weight.dtype and (
        bias is None or bias.dtype == input.dtype
    ), "Incompatible dtypes"
    assert input.shape[1] == weight.shape[0], "Incompatible input channels"
    assert input.shape[1] % groups == 0, "input channels must be divisible by groups"
    assert input.dtype in _lib.DTYPE_CODE, f"unsupported dtype: {input.dtype}"
    if not input.is_cuda:
        raise AssertionError("batch-invariant operators require CUDA tensors")
    stride = _expand(stride, nd, "stride")
    padding = _expand(padding, nd, "padding")
    dilation = _expand(dilation, nd, "dilation")
    output_padding = _expand(output_padding, nd, "output_padding")
    ksize = tuple(weight.shape[2:])
    label = "ConvTranspose2d" if nd == 2 else "ConvTranspose3d"
    assert stride == ksize, (
        f"batch-invariant {label} currently requires non-overlapping "
        f"stride == kernel_size, got stride={stride}, kernel_size={ksize}"
    )
    assert padding == (0,) * nd, f"padding is not supported, got {padding}"
    assert output_padding == (0,) * nd, f"output_padding is not supported, got {output_padding}"
    assert dilation == (1,) * nd, f"dilation is not supported, got {dilation}"

    og = weight.shape[1]
    cout = og * groups
    if bias is not None:
        assert bias.shape == (cout,), "Incompatible bias shape"
    spatial = tuple(input.shape[2:])
    out_shape = tuple(spatial[i] * ksize[i] for i in range(nd))
    batch, cin = input.shape[:2]
    out = torch.empty((batch, cout, *out_shape), device=input.device, dtype=input.dtype)
    if batch == 0 or out.numel() == 0:
        return out
    cg = cin // groups
    kvol = math.prod(ksize)
    q = og * kvol
    p = math.prod(spatial)
    x = input.contiguous()
    w = weight.contiguous()
    geom = _geom(batch, cin, groups, spatial, ksize, ksize, (0,) * nd, (1,) * nd, spatial)
    bias_c = bias.contiguous() if bias is not None else None
    if input.dtype != torch.float32 and cg > 0 and p % 8 == 0 and q % 8 == 0:
        # one GEMM whose epilogue adds the bias and writes the final layout
        st = _lib.load().bio_conv_transpose(
            _lib.DTYPE_CODE[input.dtype],
            ctypes.c_void_p(x.data_ptr()),
            ctypes.c_void_p(w.data_ptr()),
            ctypes.c_void_p(bias_c.data_ptr() if bias_c is not None else 0),
            ctypes.c_void_p(out.data_ptr()),
            ctypes.byref(geom),
            og,
            input.device.index,
            _lib.stream_of(input),
        )
        if st != _lib.BIO_ERR_ALIGN:
            _lib.check(st, "bio_conv_transpose")
            return out
    tmp = torch.empty((batch, groups, q, p), device=input.device, dtype=input.dtype)
    # A[m=q, k=c] = W[g*Cg + c, q]  (M-contiguous);  B[k=c, n=i] = X[b, g*Cg + c, i]
    opa = _gemm.operand_a(w, batch, groups, q, cg, 1, q, 0, cg * q)
    opb = _gemm.operand_b(x, batch, groups, cg, p, p, 1, cin * p, cg * p)
    if cg > 0:
        _gemm.launch(
            opa,
            opb,
            tmp,
            batch1=batch,
            batch2=groups,
            m=q,
            n=p,
            k=cg,
            c_sm=p,
            c_sn=1,
            c_s1=groups * q * p,
            c_s2=q * p,
        )
    else:
        tmp.zero_()
    _lib.check(
        _lib.load().bio_conv_transpose_scatter(
            _lib.DTYPE_CODE[input.dtype],
            ctypes.c_void_p(tmp.data_ptr()),
            ctypes.c_void_p(bias_c.data_ptr() if bias_c is not None else 0),
            ctypes.c_void_p(out.data_ptr()),
            ctypes.byref(geom),
            og,
            input.device.index,
            _lib.stream_of(input),
        ),
        "bio_conv_transpose_scatter",
    )
    return out
