"""GPU parity and batch-invariance tests of the non-GEMM operators:
convolutions, softmax / log-softmax, mean, vector norm, SDPA, varlen
attention and the MoE.  Cases mirror test_batch_invariance.py:175-780 of the
reference suite; every op is also checked against the reference's golden
vectors (tests/golden) and the fp64 oracle.
"""

from __future__ import annotations

import math
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from batch_invariant_ops import (
    _lib,
    conv1d_batch_invariant,
    conv2d_batch_invariant,
    conv3d_batch_invariant,
    conv_transpose2d_batch_invariant,
    conv_transpose3d_batch_invariant,
    deterministic_token_choice_moe,
    linalg_vector_norm_batch_invariant,
    log_softmax,
    mean_dim,
    scaled_dot_product_attention_batch_invariant,
    softmax,
    varlen_scaled_dot_product_attention_batch_invariant,
)
from batch_invariant_ops.batch_invariant_ops import convolution_batch_invariant
from conftest import DTYPES, TOLERANCES, assert_first_sample_equal
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _rn(*shape, dtype=torch.float32, gen):
    return torch.randn(*shape, device="cuda", generator=gen).to(dtype)


def _golden(name):
    case = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    return case, {k: v.cuda() for k, v in case["inputs"].items()}


def _close_to_oracle(out, ref, dtype, **override):
    tol = dict(TOLERANCES[dtype])
    tol.update(override)
    torch.testing.assert_close(out.double().cpu(), ref, **tol)


# ------------------------------------------------------------------ convolution
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("composition", ("duplicate", "unrelated"))
@pytest.mark.parametrize("batch_size", (2, 5, 17, 32))
def test_siglip_patch_conv_is_batch_invariant(dtype, composition, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(5000 + batch_size)
    target = _rn(1, 3, 28, 28, dtype=dtype, gen=gen)
    if composition == "duplicate":
        inputs = target.expand(batch_size, -1, -1, -1).contiguous()
    else:
        inputs = torch.cat((target, _rn(batch_size - 1, 3, 28, 28, dtype=dtype, gen=gen)))
    weight = _rn(32, 3, 14, 14, dtype=dtype, gen=gen)
    bias = _rn(32, dtype=dtype, gen=gen)
    args = (weight, bias, (14, 14), (0, 0), (1, 1), False, (0, 0), 1)
    assert_first_sample_equal(conv2d_batch_invariant(target, *args), conv2d_batch_invariant(inputs, *args))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 5, 17))
def test_depthwise_conv1d_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(5800 + batch_size)
    target = _rn(1, 32, 73, dtype=dtype, gen=gen)
    inputs = torch.cat((target, _rn(batch_size - 1, 32, 73, dtype=dtype, gen=gen)))
    weight = _rn(32, 1, 4, dtype=dtype, gen=gen)
    bias = _rn(32, dtype=dtype, gen=gen)
    args = (weight, bias, (1,), (3,), (1,), False, (0,), 32)
    assert_first_sample_equal(conv1d_batch_invariant(target, *args), conv1d_batch_invariant(inputs, *args))


CONV_CASES = [
    ("conv1d", (3, 4, 19), (7, 4, 3), (1,), (0,), (1,), 1),
    ("conv1d", (2, 8, 23), (12, 2, 4), (2,), (3,), (2,), 4),
    ("conv1d", (2, 16, 31), (16, 1, 4), (1,), (3,), (1,), 16),
    ("conv2d", (3, 4, 13, 11), (7, 4, 3, 3), (1, 1), (0, 0), (1, 1), 1),
    ("conv2d", (2, 4, 13, 11), (6, 2, 3, 2), (2, 1), (1, 0), (2, 1), 2),
    ("conv2d", (2, 4, 9, 9), (4, 1, 3, 3), (1, 1), (1, 1), (1, 1), 4),
    ("conv3d", (3, 3, 2, 16, 16), (12, 3, 2, 16, 16), (2, 16, 16), (0, 0, 0), (1, 1, 1), 1),
    ("conv3d", (2, 4, 7, 9, 8), (6, 2, 3, 2, 2), (2, 1, 2), (1, 0, 1), (2, 1, 1), 2),
]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: f"{c[0]}-{c[1]}-{c[2]}")
def test_conv_matches_torch_and_oracle(dtype, case):
    kind, shape, wshape, stride, padding, dilation, groups = case
    gen = torch.Generator(device="cuda").manual_seed(6000)
    x = _rn(*shape, dtype=dtype, gen=gen)
    w = _rn(*wshape, dtype=dtype, gen=gen)
    b = _rn(wshape[0], dtype=dtype, gen=gen)
    fn = {"conv1d": conv1d_batch_invariant, "conv2d": conv2d_batch_invariant,
          "conv3d": conv3d_batch_invariant}[kind]
    out = fn(x, w, b, stride, padding, dilation, False, (0,) * len(stride), groups)
    torch_fn = {"conv1d": F.conv1d, "conv2d": F.conv2d, "conv3d": F.conv3d}[kind]
    tol = {"rtol": 5e-4, "atol": 4e-2} if (kind == "conv3d" and dtype == torch.float32) else {}
    torch.testing.assert_close(out, torch_fn(x, w, b, stride, padding, dilation, groups),
                               **(tol or TOLERANCES[dtype]))
    _close_to_oracle(out, O.conv(x, w, b, stride, padding, dilation, groups), dtype, **tol)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 5, 17))
def test_qwen_patch_conv3d_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(6700 + batch_size)
    target = _rn(1, 3, 2, 16, 16, dtype=dtype, gen=gen)
    inputs = torch.cat((target, _rn(batch_size - 1, 3, 2, 16, 16, dtype=dtype, gen=gen)))
    weight = _rn(12, 3, 2, 16, 16, dtype=dtype, gen=gen)
    bias = _rn(12, dtype=dtype, gen=gen)
    args = (weight, bias, (2, 16, 16), (0, 0, 0), (1, 1, 1), False, (0, 0, 0), 1)
    assert_first_sample_equal(conv3d_batch_invariant(target, *args), conv3d_batch_invariant(inputs, *args))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("groups", (1, 2))
def test_conv_transpose_matches_torch(dtype, groups):
    gen = torch.Generator(device="cuda").manual_seed(6725 + groups)
    x2 = _rn(2, 4, 3, 3, dtype=dtype, gen=gen)
    w2 = _rn(4, 6 // groups, 2, 2, dtype=dtype, gen=gen)
    b = _rn(6, dtype=dtype, gen=gen)
    out2 = conv_transpose2d_batch_invariant(x2, w2, b, (2, 2), (0, 0), (1, 1), (0, 0), groups)
    torch.testing.assert_close(out2, F.conv_transpose2d(x2, w2, b, stride=2, groups=groups),
                               **TOLERANCES[dtype])
    x3 = _rn(2, 4, 2, 3, 3, dtype=dtype, gen=gen)
    w3 = _rn(4, 6 // groups, 2, 2, 2, dtype=dtype, gen=gen)
    out3 = conv_transpose3d_batch_invariant(x3, w3, b, (2, 2, 2), (0, 0, 0), (1, 1, 1), (0, 0, 0), groups)
    torch.testing.assert_close(out3, F.conv_transpose3d(x3, w3, b, stride=2, groups=groups),
                               **TOLERANCES[dtype])
    _close_to_oracle(out3, O.conv_transpose(x3, w3, b, (2, 2, 2), groups), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 5, 17))
def test_conv_transpose_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(6775 + batch_size)
    x = _rn(batch_size, 8, 3, 3, dtype=dtype, gen=gen)
    w = _rn(8, 6, 4, 4, dtype=dtype, gen=gen)
    b = _rn(6, dtype=dtype, gen=gen)
    args = (w, b, (4, 4), (0, 0), (1, 1), (0, 0), 1)
    assert_first_sample_equal(conv_transpose2d_batch_invariant(x[:1], *args),
                              conv_transpose2d_batch_invariant(x, *args))
    x3 = _rn(batch_size, 8, 2, 3, 3, dtype=dtype, gen=gen)
    w3 = _rn(8, 6, 4, 1, 1, dtype=dtype, gen=gen)
    args3 = (w3, b, (4, 1, 1), (0, 0, 0), (1, 1, 1), (0, 0, 0), 1)
    assert_first_sample_equal(conv_transpose3d_batch_invariant(x3[:1], *args3),
                              conv_transpose3d_batch_invariant(x3, *args3))


@pytest.mark.parametrize("name", ["conv1d_dense", "conv1d_grouped", "conv1d_depthwise", "conv2d_dense",
                                  "conv2d_grouped", "conv2d_patch14", "conv3d_patch", "conv3d_grouped",
                                  "convT2d_g1", "convT2d_g2", "convT3d_g2", "convT3d_411"])
def test_conv_matches_reference_golden(name):
    case, x = _golden(name)
    kw = case["kwargs"]
    nd = x["weight"].ndim - 2
    if case["op"] == "conv":
        out = convolution_batch_invariant(x["x"], x["weight"], x["bias"], kw["stride"], kw["padding"],
                                          kw["dilation"], False, (0,) * nd, kw["groups"])
    else:
        out = convolution_batch_invariant(x["x"], x["weight"], x["bias"], kw["stride"], (0,) * nd,
                                          (1,) * nd, True, (0,) * nd, kw["groups"])
    tol = {"rtol": 5e-4, "atol": 4e-2} if name.startswith("conv3d") else TOLERANCES[torch.float32]
    torch.testing.assert_close(out.cpu(), case["output"], **tol)


def test_conv_rejects_unsupported_geometry():
    x = torch.randn(1, 4, 6, 6, device="cuda")
    w = torch.randn(4, 2, 3, 3, device="cuda")
    with pytest.raises(AssertionError, match="stride == kernel_size"):
        conv_transpose2d_batch_invariant(x, w, None, (2, 2), (0, 0), (1, 1), (0, 0), 1)
    with pytest.raises(AssertionError, match="transposed convolution is not supported"):
        conv2d_batch_invariant(x, w.transpose(0, 1).contiguous(), None, (1, 1), (0, 0), (1, 1), True,
                               (0, 0), 1)


# ------------------------------------------------------------------ softmax family
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dim", (-1, 1))
def test_softmax_and_log_softmax_match_torch(dtype, dim):
    gen = torch.Generator(device="cuda").manual_seed(7040 + dim)
    x = _rn(3, 7, 145, dtype=dtype, gen=gen)
    torch.testing.assert_close(softmax(x, dim), torch.softmax(x, dim=dim), **TOLERANCES[dtype])
    torch.testing.assert_close(log_softmax(x, dim), torch.log_softmax(x, dim=dim), **TOLERANCES[dtype])
    _close_to_oracle(softmax(x, dim), O.softmax(x, dim), dtype)
    _close_to_oracle(log_softmax(x, dim), O.log_softmax(x, dim), dtype)


# Widths cover every row-mode kernel: one warp per row (n <= 2048), one CTA
# per row with the row in registers (n <= 16384), a cluster of 2/4/8 CTAs per
# row (n <= 262144) and the three-pass CTA kernel beyond; odd widths make
# rows start off 16-byte boundaries (element loads and stores).
@pytest.mark.parametrize("n", (1, 7, 145, 2048, 2049, 4096, 16384, 16385, 40000, 65536, 65537,
                               70001, 131073, 257152, 262144, 262145, 300001))
def test_softmax_row_widths_bitwise_invariant(n):
    gen = torch.Generator(device="cuda").manual_seed(n)
    x = _rn(9, n, dtype=torch.bfloat16, gen=gen)
    full = softmax(x, -1)
    assert torch.equal(softmax(x[:1], -1), full[:1])
    assert torch.equal(softmax(x[3:4], -1), full[3:4])
    lf = log_softmax(x, -1)
    assert torch.equal(log_softmax(x[:1], -1), lf[:1])
    assert torch.equal(log_softmax(x[5:8], -1), lf[5:8])
    _close_to_oracle(full[:2], O.softmax(x[:2], -1), torch.bfloat16)
    _close_to_oracle(lf[7:], O.log_softmax(x[7:], -1), torch.bfloat16)


@pytest.mark.parametrize("dtype", (torch.float32, torch.float16))
@pytest.mark.parametrize("n", (30000, 100003, 257152))
def test_softmax_cluster_rows_other_dtypes(dtype, n):
    gen = torch.Generator(device="cuda").manual_seed(n + 3)
    x = _rn(5, n, dtype=dtype, gen=gen) * 4
    x[1, ::3] = -math.inf
    full = softmax(x, -1)
    assert torch.equal(softmax(x[1:2], -1), full[1:2])
    _close_to_oracle(full, O.softmax(x, -1), dtype)
    lf = log_softmax(x[2:], -1)
    assert torch.equal(log_softmax(x[4:], -1), lf[2:])
    _close_to_oracle(lf, O.log_softmax(x[2:], -1), dtype)
    up = softmax(x, -1, dtype=torch.float32) if dtype != torch.float32 else full
    _close_to_oracle(up, O.softmax(x, -1), torch.float32)


def test_softmax_fully_masked_row_is_zero_and_output_dtype():
    x = torch.randn(4, 300, device="cuda")
    x[2] = -math.inf
    out = softmax(x, -1, dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    assert torch.count_nonzero(out[2]) == 0
    torch.testing.assert_close(out[0].float().sum(), torch.tensor(1.0, device="cuda"), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("name", ["softmax_f32_d1", "softmax_f32_d2", "log_softmax_f32_d1",
                                  "log_softmax_f32_d2", "softmax_bf16_d1", "softmax_bf16_d2",
                                  "log_softmax_bf16_d1", "log_softmax_bf16_d2",
                                  "softmax_f32_wide_neginf_row"])
def test_softmax_matches_reference_golden(name):
    case, x = _golden(name)
    fn = log_softmax if case["op"] == "log_softmax" else softmax
    out = fn(x["x"], case["kwargs"]["dim"])
    torch.testing.assert_close(out.cpu(), case["output"], **TOLERANCES[case["output"].dtype],
                               equal_nan=True)


# ------------------------------------------------------------------ reductions
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dimensions", ((1,), (1, 3), None))
@pytest.mark.parametrize("keepdim", (False, True))
def test_vector_norm_matches_torch(dtype, dimensions, keepdim):
    gen = torch.Generator(device="cuda").manual_seed(7050)
    x = _rn(3, 17, 5, 11, dtype=dtype, gen=gen)
    out = linalg_vector_norm_batch_invariant(x, dim=dimensions, keepdim=keepdim)
    torch.testing.assert_close(out, torch.linalg.vector_norm(x, dim=dimensions, keepdim=keepdim),
                               **TOLERANCES[dtype])
    _close_to_oracle(out, O.vector_norm(x, dimensions, keepdim), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dim", (0, 1, -1))
@pytest.mark.parametrize("keepdim", (False, True))
def test_mean_dim_matches_torch(dtype, dim, keepdim):
    gen = torch.Generator(device="cuda").manual_seed(7060)
    x = _rn(6, 33, 2048, dtype=dtype, gen=gen)
    out = mean_dim(x, dim, keepdim=keepdim)
    torch.testing.assert_close(out, x.mean(dim=dim, keepdim=keepdim), **TOLERANCES[dtype])
    _close_to_oracle(out, O.mean(x, (dim % 3,), keepdim), dtype)


def test_mean_rms_rows_bitwise_invariant():
    gen = torch.Generator(device="cuda").manual_seed(7070)
    x = _rn(64, 1, 2048, dtype=torch.bfloat16, gen=gen)
    full = mean_dim(x * x, -1, keepdim=True)
    assert torch.equal(mean_dim(x[:1] * x[:1], -1, keepdim=True), full[:1])


@pytest.mark.parametrize("name", ["mean_last", "mean_mid", "norm_1", "norm_13", "norm_0123"])
def test_reductions_match_reference_golden(name):
    case, x = _golden(name)
    dims = case["kwargs"]["dims"]
    if case["op"] == "mean":
        out = mean_dim(x["x"], dims[0])
    else:
        out = linalg_vector_norm_batch_invariant(x["x"], dim=dims)
    torch.testing.assert_close(out.cpu(), case["output"], rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 3, 5, 17))
def test_sdpa_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(7100 + batch_size)
    target = _rn(1, 16, 256, 72, dtype=dtype, gen=gen)
    query = torch.cat((target, _rn(batch_size - 1, 16, 256, 72, dtype=dtype, gen=gen)))
    key = _rn(*query.shape, dtype=dtype, gen=gen)
    value = _rn(*query.shape, dtype=dtype, gen=gen)
    alone = scaled_dot_product_attention_batch_invariant(query[:1], key[:1], value[:1])
    batched = scaled_dot_product_attention_batch_invariant(query, key, value)
    assert_first_sample_equal(alone, batched)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("causal", (False, True))
def test_sdpa_matches_torch_and_oracle(dtype, causal):
    gen = torch.Generator(device="cuda").manual_seed(7200)
    q = _rn(2, 8, 33, 65, dtype=dtype, gen=gen)
    k = _rn(2, 8, 47, 65, dtype=dtype, gen=gen)
    v = _rn(2, 8, 47, 39, dtype=dtype, gen=gen)
    out = scaled_dot_product_attention_batch_invariant(q, k, v, is_causal=causal)
    torch.testing.assert_close(out, F.scaled_dot_product_attention(q, k, v, is_causal=causal),
                               **TOLERANCES[dtype])
    _close_to_oracle(out, O.sdpa(q, k, v, None, causal), dtype)


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("head_dim", (52, 72, 100))
def test_sdpa_two_tile_head_dims_below_padded_width(head_dim, dtype):
    # more than 128 query rows and equal padded widths take the two-tile kernel;
    # 52 and 100 end in a partial group of 8 output columns (16-byte stores
    # for the aligned groups, element stores for the rest, both dtypes)
    gen = torch.Generator(device="cuda").manual_seed(7230 + head_dim)
    q = _rn(3, 2, 300, head_dim, dtype=dtype, gen=gen)
    k = _rn(3, 2, 300, head_dim, dtype=dtype, gen=gen)
    v = _rn(3, 2, 300, head_dim, dtype=dtype, gen=gen)
    out = scaled_dot_product_attention_batch_invariant(q, k, v)
    torch.testing.assert_close(out, F.scaled_dot_product_attention(q, k, v), **TOLERANCES[dtype])
    _close_to_oracle(out, O.sdpa(q, k, v, None, False), dtype)
    alone = scaled_dot_product_attention_batch_invariant(q[:1], k[:1], v[:1])
    assert_first_sample_equal(alone, out)


@pytest.mark.parametrize("mask_kind", ("boolean", "additive"))
def test_sdpa_matches_torch_with_mask(mask_kind):
    gen = torch.Generator(device="cuda").manual_seed(7250)
    q = _rn(2, 4, 17, 32, dtype=torch.bfloat16, gen=gen)
    k = _rn(2, 4, 23, 32, dtype=torch.bfloat16, gen=gen)
    v = _rn(2, 4, 23, 24, dtype=torch.bfloat16, gen=gen)
    keep = torch.rand(2, 1, 17, 23, device="cuda", generator=gen) > 0.2
    keep[:, :, -1] = False
    mask = keep if mask_kind == "boolean" else torch.where(
        keep, torch.tensor(0.0, device="cuda", dtype=torch.bfloat16),
        torch.tensor(float("-inf"), device="cuda", dtype=torch.bfloat16))
    out = scaled_dot_product_attention_batch_invariant(q, k, v, attn_mask=mask)
    expected = O.sdpa(q, k, v, mask)
    _close_to_oracle(out, expected, torch.bfloat16)
    assert torch.count_nonzero(out[:, :, -1]) == 0


def test_sdpa_grouped_query_attention():
    gen = torch.Generator(device="cuda").manual_seed(7275)
    q = _rn(2, 8, 17, 32, dtype=torch.bfloat16, gen=gen)
    k = _rn(2, 2, 23, 32, dtype=torch.bfloat16, gen=gen)
    v = _rn(2, 2, 23, 24, dtype=torch.bfloat16, gen=gen)
    out = scaled_dot_product_attention_batch_invariant(q, k, v, enable_gqa=True)
    torch.testing.assert_close(out, F.scaled_dot_product_attention(q, k, v, enable_gqa=True),
                               **TOLERANCES[torch.bfloat16])


@pytest.mark.parametrize("name", ["sdpa_causal0", "sdpa_causal1", "sdpa_boolmask", "sdpa_floatmask", "sdpa_gqa"])
def test_sdpa_matches_reference_golden(name):
    case, x = _golden(name)
    kw = case["kwargs"]
    out = scaled_dot_product_attention_batch_invariant(
        x["q"], x["k"], x["v"], attn_mask=x.get("attn_mask"), is_causal=kw.get("is_causal", False),
        scale=kw.get("scale"), enable_gqa=kw.get("enable_gqa", False))
    torch.testing.assert_close(out.cpu(), case["output"], **TOLERANCES[torch.float32])


@pytest.mark.parametrize("name", ["varlen_none", "varlen_TopLeft", "varlen_BottomRight", "varlen_uncovered",
                                  "varlen_empty_kv"])
def test_varlen_matches_reference_golden(name):
    case, x = _golden(name)
    kw = case["kwargs"]
    out = varlen_scaled_dot_product_attention_batch_invariant(
        x["q"], x["k"], x["v"], x["cu_q"], x["cu_kv"], is_causal=kw.get("is_causal", False),
        causal_type=kw.get("causal_type"))
    torch.testing.assert_close(out.cpu(), case["output"], **TOLERANCES[torch.float32])


def _offsets(lengths):
    out = [0]
    for n in lengths:
        out.append(out[-1] + n)
    return torch.tensor(out, device="cuda", dtype=torch.int32)


@pytest.mark.parametrize("causal_type", (None, "TopLeft", "BottomRight"))
def test_varlen_matches_independent_calls(causal_type):
    gen = torch.Generator(device="cuda").manual_seed(7350)
    ql, kl = (5, 3, 7), (7, 4, 5)
    q = _rn(1, sum(ql), 4, 32, dtype=torch.bfloat16, gen=gen)
    k = _rn(1, sum(kl), 2, 32, dtype=torch.bfloat16, gen=gen)
    v = _rn(1, sum(kl), 2, 24, dtype=torch.bfloat16, gen=gen)
    out = varlen_scaled_dot_product_attention_batch_invariant(
        q, k, v, _offsets(ql), _offsets(kl), is_causal=causal_type is not None, causal_type=causal_type)
    ref = O.varlen_sdpa(q, k, v, _offsets(ql), _offsets(kl), causal_type is not None, causal_type)
    _close_to_oracle(out, ref, torch.bfloat16)


def test_varlen_is_batch_invariant_for_packs():
    gen = torch.Generator(device="cuda").manual_seed(7375)
    ql, kl = (33, 17, 33), (47, 23, 47)
    q = _rn(1, sum(ql), 8, 64, dtype=torch.bfloat16, gen=gen)
    k = _rn(1, sum(kl), 8, 64, dtype=torch.bfloat16, gen=gen)
    v = _rn(1, sum(kl), 8, 64, dtype=torch.bfloat16, gen=gen)
    alone = varlen_scaled_dot_product_attention_batch_invariant(
        q[:, :33], k[:, :47], v[:, :47], _offsets(ql[:1]), _offsets(kl[:1]), is_causal=True,
        causal_type="BottomRight")
    packed = varlen_scaled_dot_product_attention_batch_invariant(
        q, k, v, _offsets(ql), _offsets(kl), is_causal=True, causal_type="BottomRight")
    assert torch.equal(alone, packed[:, :33])


def test_varlen_uncovered_rows_and_empty_kv_are_zero():
    q = torch.randn(1, 11, 2, 16, device="cuda", dtype=torch.float16)
    out = varlen_scaled_dot_product_attention_batch_invariant(
        q, torch.randn_like(q), torch.randn_like(q),
        torch.tensor([0, 5, 9], device="cuda", dtype=torch.int32),
        torch.tensor([0, 5, 9], device="cuda", dtype=torch.int32))
    assert torch.count_nonzero(out[:, :9]) > 0 and torch.count_nonzero(out[:, 9:]) == 0
    q2 = torch.randn(1, 2, 2, 16, device="cuda", dtype=torch.float16)
    k2 = torch.empty(1, 0, 2, 16, device="cuda", dtype=torch.float16)
    out2 = varlen_scaled_dot_product_attention_batch_invariant(
        q2, k2, torch.empty_like(k2), torch.tensor([0, 2], device="cuda", dtype=torch.int32),
        torch.tensor([0, 0], device="cuda", dtype=torch.int32))
    assert torch.count_nonzero(out2) == 0


# ------------------------------------------------------------------ MoE
def test_moe_matches_route_reference_and_golden():
    case, x = _golden("moe_f32")
    out = deterministic_token_choice_moe(x["hidden"], x["routing_weights"], x["selected_experts"],
                                         x["gate"], x["up"], x["down"])
    torch.testing.assert_close(out.cpu(), case["output"], rtol=2e-5, atol=2e-5)
    again = deterministic_token_choice_moe(x["hidden"], x["routing_weights"], x["selected_experts"],
                                           x["gate"], x["up"], x["down"])
    assert torch.equal(out, again)
    ref = O.moe(x["hidden"], x["routing_weights"], x["selected_experts"], x["gate"], x["up"], x["down"])
    torch.testing.assert_close(out.double().cpu(), ref, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("dtype", DTYPES)
def test_moe_is_batch_invariant(dtype):
    gen = torch.Generator(device="cuda").manual_seed(7425)
    hidden = _rn(11, 64, dtype=dtype, gen=gen)
    gate = _rn(7, 80, 64, dtype=dtype, gen=gen)
    up = _rn(7, 80, 64, dtype=dtype, gen=gen)
    down = _rn(7, 64, 80, dtype=dtype, gen=gen)
    sel = torch.randint(0, 7, (11, 4), device="cuda", generator=gen)
    w = torch.rand(11, 4, device="cuda", generator=gen)
    alone = deterministic_token_choice_moe(hidden[:1], w[:1], sel[:1], gate, up, down)
    together = deterministic_token_choice_moe(hidden, w, sel, gate, up, down)
    assert torch.equal(alone, together[:1])
    ref = O.moe(hidden, w, sel, gate, up, down)
    if dtype == torch.float32:
        err = (together.double().cpu() - ref).abs().max() / ref.abs().max()
        assert err < 2e-4, err
    else:  # normwise bar of the 16-bit contract
        err = (together.double().cpu() - ref).norm() / ref.norm()
        assert err <= 1e-2, err


def test_moe_out_of_range_expert_sets_status_not_trap():
    hidden = torch.randn(3, 16, device="cuda")
    gate = torch.randn(2, 8, 16, device="cuda")
    down = torch.randn(2, 16, 8, device="cuda")
    sel = torch.tensor([[0, 1], [1, 5], [0, 0]], device="cuda")
    w = torch.rand(3, 2, device="cuda")
    out = deterministic_token_choice_moe(hidden, w, sel, gate, gate, down)
    assert _lib.device_status() & _lib.BIO_DEV_INDEX
    assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[0]) > 0
    _lib.clear_device_status()


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_column_mode_vectorised_reductions(dtype):
    """Reductions over a non-last dim with inner % 8 == 0 (8 columns per thread)."""
    gen = torch.Generator(device="cuda").manual_seed(7080)
    x = _rn(3, 40, 4, 48, dtype=dtype, gen=gen)  # dim 1 reduced, inner = 192
    _close_to_oracle(softmax(x, 1), O.softmax(x, 1), dtype)
    _close_to_oracle(log_softmax(x, 1), O.log_softmax(x, 1), dtype)
    _close_to_oracle(mean_dim(x, 1), O.mean(x, (1,)), dtype)
    _close_to_oracle(linalg_vector_norm_batch_invariant(x, dim=1), O.vector_norm(x, (1,)), dtype)
    assert torch.equal(softmax(x[:1], 1), softmax(x, 1)[:1])
    assert torch.equal(linalg_vector_norm_batch_invariant(x[:1], dim=1),
                       linalg_vector_norm_batch_invariant(x, dim=1)[:1])


def _convt_two_step(x, w, b, k, groups):
    """The buffered path: GEMM into [B, G, Og*kvol, P], then the layout kernel."""
    import ctypes
    import math

    from batch_invariant_ops import _conv, _gemm

    nd = x.ndim - 2
    batch, cin = x.shape[:2]
    og = w.shape[1]
    cg = cin // groups
    kvol = math.prod(k)
    q, p = og * kvol, math.prod(x.shape[2:])
    out = torch.empty((batch, og * groups, *(s * kk for s, kk in zip(x.shape[2:], k))),
                      device="cuda", dtype=x.dtype)
    tmp = torch.empty((batch, groups, q, p), device="cuda", dtype=x.dtype)
    xc, wc = x.contiguous(), w.contiguous()
    opa = _gemm.operand_a(wc, batch, groups, q, cg, 1, q, 0, cg * q)
    opb = _gemm.operand_b(xc, batch, groups, cg, p, p, 1, cin * p, cg * p)
    _gemm.launch(opa, opb, tmp, batch1=batch, batch2=groups, m=q, n=p, k=cg, c_sm=p, c_sn=1,
                 c_s1=groups * q * p, c_s2=q * p)
    geom = _conv._geom(batch, cin, groups, tuple(x.shape[2:]), k, k, (0,) * nd, (1,) * nd,
                       tuple(x.shape[2:]))
    _lib.check(_lib.load().bio_conv_transpose_scatter(
        _lib.DTYPE_CODE[x.dtype], ctypes.c_void_p(tmp.data_ptr()),
        ctypes.c_void_p(b.data_ptr() if b is not None else 0), ctypes.c_void_p(out.data_ptr()),
        ctypes.byref(geom), og, 0, _lib.stream_of(x)), "bio_conv_transpose_scatter")
    return out


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
@pytest.mark.parametrize(
    "shape,cout,k,groups,with_bias",
    [((8, 256, 24, 24), 256, (4, 4), 1, True), ((3, 64, 16, 16), 32, (2, 2), 2, False),
     ((2, 32, 8, 16), 48, (3, 3), 1, True), ((2, 64, 4, 8), 16, (16, 16), 1, True),
     ((2, 16, 4, 4, 8), 24, (2, 2, 2), 1, True), ((1, 96, 7, 9), 63, (4, 4), 3, True),
     ((5, 40, 16, 32), 8, (1, 8), 1, False)],
)
def test_fused_conv_transpose_epilogue(dtype, shape, cout, k, groups, with_bias):
    """The scatter epilogue (one GEMM writing the final layout) equals the
    buffered GEMM + layout kernel, the oracle and stock torch; shapes with
    odd sizes take the buffered path and must agree too."""
    gen = torch.Generator(device="cuda").manual_seed(sum(shape) + cout)
    x = _rn(*shape, dtype=dtype, gen=gen)
    w = (_rn(shape[1], cout // groups, *k, gen=gen) * 0.05).to(dtype)
    b = _rn(cout, dtype=dtype, gen=gen) if with_bias else None
    nd = len(k)
    fn = conv_transpose2d_batch_invariant if nd == 2 else conv_transpose3d_batch_invariant
    out = fn(x, w, b, k, (0,) * nd, (1,) * nd, (0,) * nd, groups)
    assert torch.equal(out, _convt_two_step(x, w, b, k, groups))
    assert torch.equal(fn(x[:1], w, b, k, (0,) * nd, (1,) * nd, (0,) * nd, groups), out[:1])
    tfn = F.conv_transpose2d if nd == 2 else F.conv_transpose3d
    torch.testing.assert_close(out, tfn(x, w, b, stride=k, groups=groups), **TOLERANCES[dtype])


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
@pytest.mark.parametrize("n", (16392, 40000, 65536, 131072, 257152, 262144))
@pytest.mark.parametrize("log", (False, True))
def test_cluster_softmax_register_forms_agree(dtype, n, log):
    """Long rows: aligned 16-bit rows keep raw words in registers, unaligned
    rows keep floats; both forms must give the same bits."""
    gen = torch.Generator(device="cuda").manual_seed(n + int(log))
    rows = 3
    buf = (torch.randn(rows * n + 8, device="cuda", generator=gen) * 4).to(dtype)
    aligned = buf[: rows * n].view(rows, n)
    unaligned = buf[1 : 1 + rows * n].view(rows, n)  # 2-byte offset
    ref_input = unaligned.clone()                   # aligned copy of the same values
    fn = log_softmax if log else softmax
    a = fn(ref_input, -1)
    b = fn(unaligned, -1)
    assert torch.equal(a, b)
    assert torch.equal(fn(aligned[1:2].clone(), -1), fn(aligned, -1)[1:2])
    ref = O.log_softmax(ref_input, -1) if log else O.softmax(ref_input, -1)
    _close_to_oracle(a, ref, dtype)
