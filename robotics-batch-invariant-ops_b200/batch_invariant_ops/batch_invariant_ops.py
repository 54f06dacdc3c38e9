"""Batch-invariant operators backed by hand-written sm_100a CUDA kernels.

Drop-in for ``batch_invariant_ops/batch_invariant_ops.py`` of
yiannisha/robotics-batch-invariant-ops: same public names, signatures,
assertion/exception types and ``torch.library`` override surface.  Every
operator here ends in the C ABI of ``libbio_sm100.so``; nothing calls Triton,
cuBLAS, cuDNN or a CPU path.  Line citations (``:NNN``) refer to that
reference file.
"""

from __future__ import annotations

import contextlib
from collections import namedtuple
from typing import Any

import torch

from . import _attn, _conv, _gemm, _lib, _rows

__all__ = [
    "set_batch_invariant_mode",
    "is_batch_invariant_mode_enabled",
    "disable_batch_invariant_mode",
    "enable_batch_invariant_mode",
    "matmul_persistent",
    "bmm_persistent",
    "conv1d_batch_invariant",
    "conv2d_batch_invariant",
    "conv3d_batch_invariant",
    "conv_transpose2d_batch_invariant",
    "conv_transpose3d_batch_invariant",
    "scaled_dot_product_attention_batch_invariant",
    "varlen_scaled_dot_product_attention_batch_invariant",
    "linalg_vector_norm_batch_invariant",
    "softmax",
]

_FLOAT_TYPES = (torch.float16, torch.bfloat16, torch.float32)


def get_compute_units() -> int:
    """SM count of the current CUDA device (reference :232-253)."""
    out = _lib.ctypes.c_int(0)
    _lib.check(_lib.load().bio_sm_count(torch.cuda.current_device(), _lib.ctypes.byref(out)),
               "bio_sm_count")
    return out.value


def _current_accelerator_type() -> str:
    """Active accelerator type (reference :256-268)."""
    accelerator = getattr(torch, "accelerator", None)
    if accelerator is not None:
        current = accelerator.current_accelerator()
        if current is not None:
            return current.type
    if torch.cuda.is_available():
        return "cuda"
    return "cpu"


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise AssertionError("batch-invariant operators require CUDA tensors")


# ---------------------------------------------------------------------------
# GEMM family (reference :271-431, :1600-1620)
# ---------------------------------------------------------------------------
def matmul_persistent(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None):
    """C = a @ b (+ bias); every output element is accumulated in a fixed K order
    that depends on nothing but K and the dtype (reference :271-343)."""
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.dtype == b.dtype, "Incompatible dtypes"
    assert (
        bias is None or bias.dim() == 1
    ), "Currently assuming bias is 1D, let Horace know if you run into this"
    assert a.dtype in _FLOAT_TYPES, f"unsupported dtype: {a.dtype}"
    _require_cuda(a, b, bias)
    return _gemm.mm(a, b, bias)


def bmm_persistent(a: torch.Tensor, b: torch.Tensor):
    """Batch-invariant ``torch.bmm``: every batch element is an independent GEMM
    with the same fixed schedule (reference :346-431)."""
    assert a.ndim == b.ndim == 3, "bmm expects two rank-3 tensors"
    assert a.shape[0] == b.shape[0] and a.shape[2] == b.shape[1], "Incompatible dimensions"
    assert a.dtype == b.dtype, "Incompatible dtypes"
    assert a.dtype in {
        torch.float16,
        torch.bfloat16,
        torch.float32,
    }, f"unsupported dtype: {a.dtype}"
    _require_cuda(a, b)
    return _gemm.bmm(a, b)


def mm_batch_invariant(a, b):
    return matmul_persistent(a, b)


def addmm_batch_invariant(bias, a, b, *, beta=1, alpha=1):
    """``aten::addmm``: beta * bias + alpha * (a @ b) (reference :1604-1605,
    which takes only the default beta = alpha = 1).  alpha scales the fp32
    accumulator before the bias add; beta * bias is formed in fp32 and
    rounded to the bias dtype once per column, the same for every row, so
    the result stays batch invariant.  beta = 0 ignores bias (as aten does)."""
    if beta == 1 and alpha == 1:
        return matmul_persistent(a, b, bias=bias)
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.dtype == b.dtype, "Incompatible dtypes"
    assert (
        bias is None or bias.dim() == 1
    ), "Currently assuming bias is 1D, let Horace know if you run into this"
    assert a.dtype in _FLOAT_TYPES, f"unsupported dtype: {a.dtype}"
    _require_cuda(a, b, bias)
    if beta == 0:
        bias = None
    elif beta != 1 and bias is not None:
        bias = (bias.float() * float(beta)).to(bias.dtype)
    return _gemm.mm(a, b, bias, alpha=float(alpha))


def linear_batch_invariant(input, weight, bias=None):
    """Batch-invariant ``aten::linear`` for arbitrary leading dimensions (reference :1608-1616)."""
    assert input.ndim >= 1, "linear input must have at least one dimension"
    assert weight.ndim == 2, "linear weight must be a matrix"
    assert input.shape[-1] == weight.shape[-1], "Incompatible dimensions"
    output_shape = (*input.shape[:-1], weight.shape[0])
    flattened = input.reshape(-1, input.shape[-1])
    output = matmul_persistent(flattened, weight.transpose(0, 1), bias=bias)
    return output.reshape(output_shape)


def gated_linear_batch_invariant(input, weight, activation="gelu_tanh"):
    """Gated linear unit in one fused GEMM: with ``weight`` [2F, K] holding the
    gate rows first, returns act(input @ weight[:F]^T) * (input @ weight[F:]^T)
    of shape [..., F] -- the ``gate, up = F.linear(input, weight).split(F, -1)``
    followed by ``F.gelu(gate, approximate="tanh") * up`` (activation
    "gelu_tanh", GeGLU) or ``F.silu(gate) * up`` ("silu", SwiGLU) of a
    transformer MLP, with the same rounding steps (gate and up rounded to the
    dtype, the activation rounded, the product rounded).  For f16/bf16 the
    gate and up accumulators share one tile of the tensor-core GEMM and the
    gate/up activations never reach HBM.  Each output row depends on its own
    input row only, so the result is batch invariant.  Not in the reference,
    which has no fused MLP operator."""
    _require_cuda(input, weight)
    if activation not in ("gelu_tanh", "silu"):
        raise ValueError(f"unsupported gated activation: {activation}")
    assert weight.ndim == 2 and weight.shape[0] % 2 == 0, "gated weight must be [2F, K]"
    assert input.shape[-1] == weight.shape[-1], "Incompatible dimensions"
    assert input.dtype == weight.dtype, "input and weight dtypes must match"
    f = weight.shape[0] // 2
    flat = input.reshape(-1, input.shape[-1])
    out = None
    if input.dtype in (torch.float16, torch.bfloat16) and flat.shape[1] > 0:
        out = _gemm.gated(flat, weight, activation == "gelu_tanh")
    if out is None:
        gate, up = linear_batch_invariant(flat, weight).split(f, dim=-1)
        act = (torch.nn.functional.gelu(gate, approximate="tanh") if activation == "gelu_tanh"
               else torch.nn.functional.silu(gate))
        out = act * up
    return out.reshape(*input.shape[:-1], f)


def linear_residual_batch_invariant(residual, input, weight, bias=None):
    """``residual + F.linear(input, weight, bias)`` in one GEMM whose epilogue
    adds the residual: the linear's output is rounded to the dtype, the
    residual added in fp32 and the sum rounded -- the bits of the two stock
    ops, without the round trip of the linear's output through HBM.  The
    residual stream of a transformer block (``x = x + proj(h)``) is the use.
    Each output row depends on its own input and residual rows only, so the
    result is batch invariant.  f16/bf16 run fused; other dtypes compose the
    library's linear with a stock add.  Not in the reference."""
    _require_cuda(residual, input, weight, bias)
    assert input.shape[-1] == weight.shape[-1], "Incompatible dimensions"
    out_shape = (*input.shape[:-1], weight.shape[0])
    assert tuple(residual.shape) == out_shape, "residual must have the linear's output shape"
    assert residual.dtype == input.dtype == weight.dtype, "residual, input and weight dtypes must match"
    flat = input.reshape(-1, input.shape[-1])
    out = None
    if input.dtype in (torch.float16, torch.bfloat16) and flat.shape[1] > 0:
        r2 = residual.reshape(-1, weight.shape[0])
        out = _gemm.linear_residual(r2, flat, weight, bias)
    if out is None:
        return residual + linear_batch_invariant(input, weight, bias)
    return out.reshape(out_shape)


def bmm_batch_invariant(a, b):
    return bmm_persistent(a, b)


# ---------------------------------------------------------------------------
# Convolution family (reference :434-971)
# ---------------------------------------------------------------------------
def conv1d_batch_invariant(
    input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
):
    """Batch-invariant 1-D convolution (reference :497-595)."""
    return _conv.conv_nd(
        input, weight, bias, stride, padding, dilation, transposed, output_padding, groups, 1
    )


def conv2d_batch_invariant(
    input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
):
    """Batch-invariant 2-D convolution (reference :598-682)."""
    return _conv.conv_nd(
        input, weight, bias, stride, padding, dilation, transposed, output_padding, groups, 2
    )


def conv3d_batch_invariant(
    input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
):
    """Batch-invariant 3-D convolution (reference :685-780)."""
    return _conv.conv_nd(
        input, weight, bias, stride, padding, dilation, transposed, output_padding, groups, 3
    )


def conv_transpose2d_batch_invariant(
    input, weight, bias, stride, padding, dilation, output_padding, groups
):
    """Non-overlapping (stride == kernel) 2-D transposed convolution (reference :783-861)."""
    return _conv.conv_transpose_nd(
        input, weight, bias, stride, padding, dilation, output_padding, groups, 2
    )


def conv_transpose3d_batch_invariant(
    input, weight, bias, stride, padding, dilation, output_padding, groups
):
    """Non-overlapping (stride == kernel) 3-D transposed convolution (reference :864-941)."""
    return _conv.conv_transpose_nd(
        input, weight, bias, stride, padding, dilation, output_padding, groups, 3
    )


def convolution_batch_invariant(
    input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
):
    """Dispatch supported regular and transposed ``aten::convolution`` calls (reference :944-971)."""
    if input.ndim == 3 and weight.ndim == 3:
        return conv1d_batch_invariant(
            input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
        )
    if input.ndim == 4 and weight.ndim == 4 and transposed:
        return conv_transpose2d_batch_invariant(
            input, weight, bias, stride, padding, dilation, output_padding, groups
        )
    if input.ndim == 4 and weight.ndim == 4:
        return conv2d_batch_invariant(
            input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
        )
    if input.ndim == 5 and weight.ndim == 5 and transposed:
        return conv_transpose3d_batch_invariant(
            input, weight, bias, stride, padding, dilation, output_padding, groups
        )
    if input.ndim == 5 and weight.ndim == 5:
        return conv3d_batch_invariant(
            input, weight, bias, stride, padding, dilation, transposed, output_padding, groups
        )
    raise AssertionError(
        f"only 1-D, 2-D and 3-D convolution are supported, got input rank {input.ndim} "
        f"and weight rank {weight.ndim}"
    )


# ---------------------------------------------------------------------------
# Row softmax family (reference :974-1145)
# ---------------------------------------------------------------------------
def log_softmax(input: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Batch-invariant log_softmax along ``dim`` (reference :1037-1071)."""
    _require_cuda(input)
    return _rows.softmax(input, dim, None, log=True)


def softmax(
    input: torch.Tensor,
    dim: int = -1,
    *,
    dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Batch-invariant softmax along an arbitrary dimension (reference :1117-1145)."""
    if input.dtype not in {torch.float16, torch.bfloat16, torch.float32}:
        raise ValueError(f"unsupported softmax dtype: {input.dtype}")
    if dtype not in {None, torch.float16, torch.bfloat16, torch.float32}:
        raise ValueError(f"unsupported softmax output dtype: {dtype}")
    _require_cuda(input)
    return _rows.softmax(input, dim, dtype, log=False)


def _half_to_float_input(input):
    assert input.dtype in {torch.float16, torch.bfloat16}, (
        "half_to_float requires a float16 or bfloat16 input"
    )


def _log_softmax_batch_invariant(input, dim, _half_to_float):
    """``aten::_log_softmax``; half_to_float (a 16-bit input with an fp32
    result, which the reference rejects, :1623-1625) stores the same fp32
    row result without the final rounding to 16 bits."""
    if _half_to_float:
        _half_to_float_input(input)
        _require_cuda(input)
        return _rows.softmax(input, dim, torch.float32, log=True)
    return log_softmax(input, dim=dim)


def _softmax_batch_invariant(input, dim, _half_to_float):
    """``aten::_softmax``; half_to_float as for _log_softmax (reference
    :1628-1630 rejects it)."""
    if _half_to_float:
        _half_to_float_input(input)
        return softmax(input, dim=dim, dtype=torch.float32)
    return softmax(input, dim=dim)


# ---------------------------------------------------------------------------
# Attention (reference :1148-1344)
# ---------------------------------------------------------------------------
def scaled_dot_product_attention_batch_invariant(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attn_mask: torch.Tensor | None = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    *,
    scale: float | None = None,
    enable_gqa: bool = False,
) -> torch.Tensor:
    """Fixed-schedule SDPA: every (batch, head, query row) is reduced
    independently over KV blocks in a fixed order (reference :1148-1213)."""
    if dropout_p != 0.0:
        raise ValueError("batch-invariant SDPA only supports dropout_p=0")
    if query.ndim < 3 or key.ndim != query.ndim or value.ndim != query.ndim:
        raise ValueError("query, key, and value must have matching rank >= 3")
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise ValueError("query, key, and value must have the same dtype")
    if query.dtype not in {torch.float16, torch.bfloat16, torch.float32}:
        raise ValueError(f"unsupported attention dtype: {query.dtype}")
    if enable_gqa:
        if query.shape[-3] % key.shape[-3] or key.shape[-3] != value.shape[-3]:
            raise ValueError("invalid grouped-query attention head counts")
    if query.shape[:-3] != key.shape[:-3] or query.shape[:-3] != value.shape[:-3]:
        raise ValueError("leading query, key, and value dimensions must match")
    if not enable_gqa and (query.shape[-3] != key.shape[-3] or query.shape[-3] != value.shape[-3]):
        raise ValueError("leading query, key, and value dimensions must match")
    if query.shape[-1] != key.shape[-1] or key.shape[-2] != value.shape[-2]:
        raise ValueError("incompatible attention dimensions")
    if is_causal and attn_mask is not None:
        raise ValueError("attn_mask and is_causal cannot both be set")
    _require_cuda(query, key, value, attn_mask)
    return _attn.sdpa(query, key, value, attn_mask, is_causal, scale)


def varlen_scaled_dot_product_attention_batch_invariant(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    cumulative_seqlen_q: torch.Tensor,
    cumulative_seqlen_kv: torch.Tensor,
    *,
    is_causal: bool = False,
    causal_type: Any | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Attention over sequence-packed ``[1, T, H, D]`` inputs; each sequence is
    evaluated independently (reference :1216-1344).  Sequence offsets are read
    on the device: there is no host synchronisation."""
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("varlen attention expects rank-4 query, key, and value")
    if query.shape[0] != 1 or key.shape[0] != 1 or value.shape[0] != 1:
        raise ValueError("varlen attention expects sequence-packed batch size 1")
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise ValueError("query, key, and value must have the same dtype")
    if key.shape[1] != value.shape[1] or key.shape[2] != value.shape[2]:
        raise ValueError("key and value token and head dimensions must match")
    if query.shape[3] != key.shape[3]:
        raise ValueError("query and key head dimensions must match")
    if key.shape[2] == 0 or query.shape[2] % key.shape[2]:
        raise ValueError("query heads must be divisible by key/value heads")
    if cumulative_seqlen_q.ndim != 1 or cumulative_seqlen_kv.ndim != 1:
        raise ValueError("cumulative sequence lengths must be rank 1")
    integer_dtypes = {torch.int32, torch.int64}
    if (
        cumulative_seqlen_q.dtype not in integer_dtypes
        or cumulative_seqlen_kv.dtype not in integer_dtypes
    ):
        raise ValueError("cumulative sequence lengths must use int32 or int64")
    if cumulative_seqlen_q.numel() != cumulative_seqlen_kv.numel():
        raise ValueError("query and KV cumulative sequence counts must match")
    if cumulative_seqlen_q.numel() == 0:
        raise ValueError("cumulative sequence lengths must start at zero")
    if query.dtype not in {torch.float16, torch.bfloat16, torch.float32}:
        raise ValueError(f"unsupported varlen attention dtype: {query.dtype}")
    causal_name = getattr(causal_type, "name", None)
    if causal_name is None and causal_type is not None:
        causal_name = str(causal_type).rsplit(".", 1)[-1]
    if causal_name not in {None, "TopLeft", "BottomRight", "DontCare"}:
        raise ValueError(f"causal type {causal_name!r} requires equal query and KV lengths")
    _require_cuda(query, key, value, cumulative_seqlen_q, cumulative_seqlen_kv)
    return _attn.varlen(
        query,
        key,
        value,
        cumulative_seqlen_q,
        cumulative_seqlen_kv,
        is_causal=is_causal,
        causal_name=causal_name,
        scale=scale,
    )


# ---------------------------------------------------------------------------
# Reductions (reference :1347-1597, :1633-1651)
# ---------------------------------------------------------------------------
def mean_dim(
    input: torch.Tensor, dim: int, keepdim: bool = False, dtype: torch.dtype | None = None
) -> torch.Tensor:
    """Mean over one dimension with a fixed per-output reduction tree (reference :1395-1482)."""
    assert input.is_cuda, "Input must be a CUDA tensor"
    assert (
        -input.ndim <= dim < input.ndim
    ), f"Invalid dimension {dim} for tensor with {input.ndim} dimensions"
    if dim < 0:
        dim = dim + input.ndim
    if dtype is None:
        if input.dtype in [torch.int8, torch.int16, torch.int32, torch.int64]:
            dtype = torch.float32
        else:
            dtype = input.dtype
    if input.dtype != dtype:
        input = input.to(dtype)
    return _rows.reduce_dims(input, (dim,), keepdim, kind="mean")


def mean_batch_invariant(input, dim, keepdim=False, dtype: torch.dtype | None = None):
    """``aten::mean.dim`` override (reference :1633-1651).  Multi-dimension means
    run on the same fixed-tree kernel (the reference falls back to stock
    ``torch.sum`` there)."""
    assert dtype is None or dtype == torch.float32, f"unsupported dtype: {dtype}"
    if dim is not None and len(dim) == 1:
        return mean_dim(input, dim[0], keepdim=keepdim)
    assert input.dtype in {
        torch.float16,
        torch.bfloat16,
        torch.float32,
    }, "only float types supported for now"
    _require_cuda(input)
    if dim is None or len(dim) == 0:
        dim = list(range(input.ndim))
    dims = tuple(sorted({d % input.ndim for d in dim}))
    out_dtype = dtype or input.dtype
    return _rows.reduce_dims(input, dims, keepdim, kind="mean", out_dtype=out_dtype)


def linalg_vector_norm_batch_invariant(
    input: torch.Tensor,
    ord: float = 2,
    dim: int | list[int] | tuple[int, ...] | None = None,
    keepdim: bool = False,
    *,
    dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Euclidean vector norm with a fixed per-vector reduction tree (reference :1525-1597)."""
    assert input.is_cuda, "input must be a CUDA tensor"
    assert input.is_floating_point(), "only real floating-point inputs are supported"
    assert float(ord) == 2.0, f"only the Euclidean norm is supported, got ord={ord!r}"
    if dtype is not None:
        assert dtype in {
            torch.float16,
            torch.bfloat16,
            torch.float32,
            torch.float64,
        }, f"unsupported dtype: {dtype}"
        assert dtype != torch.float64, "float64 is not supported by the batch-invariant kernels"
        input = input.to(dtype)
    assert input.dtype in _FLOAT_TYPES, f"unsupported dtype: {input.dtype}"
    if dim is None:
        dimensions = tuple(range(input.ndim))
    elif isinstance(dim, int):
        dimensions = (dim,)
    else:
        dimensions = tuple(dim)
    dimensions = tuple(dimension % input.ndim for dimension in dimensions) if input.ndim else ()
    assert len(set(dimensions)) == len(dimensions), "duplicate dimensions are not allowed"
    return _rows.reduce_dims(input, dimensions, keepdim, kind="l2norm")


# ---------------------------------------------------------------------------
# Fused normalisation (not in the reference; see the module docstring)
# ---------------------------------------------------------------------------
def layer_norm_batch_invariant(input, normalized_shape, weight=None, bias=None, eps=1e-5):
    """``F.layer_norm`` with a fixed per-row reduction tree: mean and biased
    variance in fp32 (two passes over the row in registers), then
    (x - mean) * rsqrt(var + eps) * weight + bias and one rounding.  The
    reference leaves layer norms to stock torch; this is the fused kernel
    its row-reduction design (mean_dim, :1395-1482) implies."""
    _require_cuda(input, weight, bias)
    return _rows.norm(input, normalized_shape, weight, bias, eps, rms=False)


def rms_norm_batch_invariant(input, normalized_shape, weight=None, eps=None):
    """``F.rms_norm`` (aten::_fused_rms_norm semantics: fp32 arithmetic,
    x * rsqrt(mean(x^2) + eps) * weight, one rounding; eps defaults to the
    fp32 machine epsilon) with a fixed per-row reduction tree.  Replaces the
    RMSNorm the reference builds from mean_dim (:1395-1482)."""
    _require_cuda(input, weight)
    if eps is None:
        eps = torch.finfo(torch.float32).eps
    return _rows.norm(input, normalized_shape, weight, None, eps, rms=True)


def native_layer_norm_batch_invariant(input, normalized_shape, weight, bias, eps):
    """``aten::native_layer_norm`` override: (output, mean, rstd), statistics
    in fp32 with shape input.shape[:-len(normalized_shape)] + (1, ...)."""
    _require_cuda(input, weight, bias)
    out, mean, rstd = _rows.norm(input, normalized_shape, weight, bias, eps, rms=False,
                                 want_stats=True)
    return out, mean, rstd


def fused_rms_norm_batch_invariant(input, normalized_shape, weight, eps):
    """``aten::_fused_rms_norm`` override: (output, rstd in fp32)."""
    _require_cuda(input, weight)
    if eps is None:
        eps = torch.finfo(torch.float32).eps
    out, _, rstd = _rows.norm(input, normalized_shape, weight, None, eps, rms=True,
                              want_stats=True)
    return out, rstd


# ---------------------------------------------------------------------------
# Mode / dispatcher override (reference :1654-1712)
# ---------------------------------------------------------------------------
_batch_invariant_MODE = False
_batch_invariant_LIB = None


def is_batch_invariant_mode_enabled():
    return _batch_invariant_MODE


def enable_batch_invariant_mode():
    """Register the batch-invariant kernels for the reference's 10 aten ops on
    the current accelerator's dispatch key (reference :1662-1684), plus the
    fused normalisations aten::native_layer_norm and aten::_fused_rms_norm
    (additions: the reference leaves normalisation to stock torch)."""
    global _batch_invariant_MODE, _batch_invariant_LIB
    if _batch_invariant_MODE:
        return
    dispatch_key = _current_accelerator_type().upper()
    _batch_invariant_MODE = True
    _batch_invariant_LIB = torch.library.Library("aten", "IMPL")
    _batch_invariant_LIB.impl("aten::mm", mm_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl("aten::addmm", addmm_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl("aten::linear", linear_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl("aten::bmm", bmm_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl("aten::convolution", convolution_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl(
        "aten::scaled_dot_product_attention",
        scaled_dot_product_attention_batch_invariant,
        dispatch_key,
    )
    _batch_invariant_LIB.impl("aten::_softmax", _softmax_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl("aten::_log_softmax", _log_softmax_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl("aten::mean.dim", mean_batch_invariant, dispatch_key)
    _batch_invariant_LIB.impl(
        "aten::linalg_vector_norm", linalg_vector_norm_batch_invariant, dispatch_key
    )
    # additions to the reference's 10 overrides: the fused normalisations
    # (F.layer_norm reaches aten::native_layer_norm, F.rms_norm on CUDA
    # aten::_fused_rms_norm)
    _batch_invariant_LIB.impl(
        "aten::native_layer_norm", native_layer_norm_batch_invariant, dispatch_key
    )
    if hasattr(torch.ops.aten, "_fused_rms_norm"):
        _batch_invariant_LIB.impl(
            "aten::_fused_rms_norm", fused_rms_norm_batch_invariant, dispatch_key
        )


def disable_batch_invariant_mode():
    """Remove the overrides (reference :1687-1692)."""
    global _batch_invariant_MODE, _batch_invariant_LIB
    if _batch_invariant_LIB is not None:
        _batch_invariant_LIB._destroy()
    _batch_invariant_MODE = False
    _batch_invariant_LIB = None


@contextlib.contextmanager
def set_batch_invariant_mode(enabled: bool = True):
    """Re-entrant, exception-safe mode switch restoring the previous state
    (reference :1695-1712)."""
    previously_enabled = is_batch_invariant_mode_enabled()
    if enabled == previously_enabled:
        yield
        return

    if enabled:
        enable_batch_invariant_mode()
    else:
        disable_batch_invariant_mode()
    try:
        yield
    finally:
        if previously_enabled:
            enable_batch_invariant_mode()
        else:
            disable_batch_invariant_mode()


AttentionBlockSize = namedtuple("AttentionBlockSize", ["block_m", "block_n"])


def get_batch_invariant_attention_block_size() -> AttentionBlockSize:
    """Constant (16, 16) block size for vLLM's attention hook (reference :1715-1719)."""
    return AttentionBlockSize(block_m=16, block_n=16)

