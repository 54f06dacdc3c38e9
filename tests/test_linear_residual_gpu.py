"""Fused linear + residual add (bio_gemm_residual).

``linear_residual_batch_invariant(r, x, w, b)`` must give the bits of the two
ops it replaces -- the library's own linear, then a stock ``r + y`` -- for
one-m-block GEMMs (single-CTA tiles, including the 96-wide one) and large
ones (CTA pairs), with and without bias, with a residual whose rows are
strided, and for B=1 against the first row of B=N; and stay within the
bf16/fp16 bar of the fp64 oracle.
"""

from __future__ import annotations

import pytest
import torch

from batch_invariant_ops import linear_batch_invariant, linear_residual_batch_invariant
from conftest import DTYPES
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
HALF = tuple(d for d in DTYPES if d != torch.float32)


def _inputs(m, k, n, dtype, seed, bias):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(dtype)
    r = torch.randn(m, n, device="cuda", generator=g).to(dtype)
    b = (0.1 * torch.randn(n, device="cuda", generator=g)).to(dtype) if bias else None
    return x, w, r, b


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("bias", (False, True))
@pytest.mark.parametrize("m,k,n", [(1, 1024, 2048), (50, 2048, 1024), (128, 4096, 11008),
                                   (400, 1152, 1152), (1600, 4096, 1024), (2000, 256, 200)])
def test_linear_residual_equals_composition(dtype, bias, m, k, n):
    x, w, r, b = _inputs(m, k, n, dtype, 11_000 + m + n, bias)
    out = linear_residual_batch_invariant(r, x, w, b)
    ref = r + linear_batch_invariant(x, w, b)
    assert torch.equal(out, ref), int((out != ref).sum())
    rows = torch.arange(0, m, max(1, m // 8), device="cuda")
    oracle = O.linear(x[rows], w, b) + r[rows].double().cpu()
    err = float((out[rows].double().cpu() - oracle).norm() / oracle.norm())
    assert err <= 1e-2, err


@pytest.mark.parametrize("dtype", HALF)
def test_linear_residual_strided_residual_and_leading_dims(dtype):
    x, w, r, b = _inputs(2 * 300, 512, 384, dtype, 12_000, True)
    wide = torch.randn(600, 512, device="cuda").to(dtype)
    wide[:, :384] = r
    rs = wide[:, :384]                      # rows 512 elements apart
    out = linear_residual_batch_invariant(rs, x, w, b)
    assert torch.equal(out, rs + linear_batch_invariant(x, w, b))
    x3, r3 = x.view(2, 300, 512), r.view(2, 300, 384)
    out3 = linear_residual_batch_invariant(r3, x3, w, b)
    assert out3.shape == (2, 300, 384)
    assert torch.equal(out3.view(600, 384), linear_residual_batch_invariant(r, x, w, b))


@pytest.mark.parametrize("dtype", HALF)
def test_linear_residual_first_row_alone_is_bitwise_equal(dtype):
    x, w, r, b = _inputs(1537, 2048, 2048, dtype, 13_000, True)
    full = linear_residual_batch_invariant(r, x, w, b)
    alone = linear_residual_batch_invariant(r[:1], x[:1], w, b)
    assert torch.equal(alone, full[:1])


def test_linear_residual_fp32_composes_and_rejects_bad_shapes():
    x, w, r, b = _inputs(33, 64, 48, torch.float32, 14_000, True)
    out = linear_residual_batch_invariant(r, x, w, b)
    assert torch.equal(out, r + linear_batch_invariant(x, w, b))
    with pytest.raises(AssertionError):
        linear_residual_batch_invariant(r[:, :40], x, w, b)
