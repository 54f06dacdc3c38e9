"""Fused gated linear (GeGLU / SwiGLU input projection, bio_gemm_swiglu).

``gated_linear_batch_invariant(x, W)`` with W = [W_gate; W_up] must give the
bits of the composition it replaces -- the library's own linear, then
``F.gelu(gate, approximate="tanh") * up`` (or ``F.silu(gate) * up``) with
stock PyTorch elementwise kernels -- and stay within the bf16/fp16 bar of the
fp64 oracle.  Checked at the VLA model's MLP shapes (prefix LM 2048 -> 2 x
16384, action expert 1024 -> 2 x 4096, small row counts of one request) and
for B=1 against the first row of B=N.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from batch_invariant_ops import gated_linear_batch_invariant, linear_batch_invariant
from conftest import DTYPES
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
HALF = tuple(d for d in DTYPES if d != torch.float32)


def _inputs(m, k, f, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    w = (torch.randn(2 * f, k, device="cuda", generator=g) / k ** 0.5).to(dtype)
    return x, w


def _composed(x, w, activation):
    gate, up = linear_batch_invariant(x, w).split(w.shape[0] // 2, dim=-1)
    act = F.gelu(gate, approximate="tanh") if activation == "gelu_tanh" else F.silu(gate)
    return act * up


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("activation", ("gelu_tanh", "silu"))
@pytest.mark.parametrize("m,k,f", [(1, 1024, 4096), (50, 1024, 4096), (300, 2048, 16384),
                                   (1000, 1024, 4096), (77, 256, 200)])
def test_gated_linear_equals_composition_and_oracle(dtype, activation, m, k, f):
    x, w = _inputs(m, k, f, dtype, 90_000 + m + f)
    out = gated_linear_batch_invariant(x, w, activation)
    ref = _composed(x, w, activation)
    assert out.shape == (m, f)
    assert torch.equal(out, ref), (
        f"fused {activation} differs from the composition in "
        f"{int((out != ref).sum())} of {out.numel()} elements")
    rows = torch.arange(0, m, max(1, m // 16), device="cuda")
    oracle = O.gated_linear(x[rows], w, activation)
    err = float((out[rows].double().cpu() - oracle).norm() / oracle.norm())
    assert err <= 1e-2, err


@pytest.mark.parametrize("dtype", HALF)
def test_gated_linear_first_row_alone_is_bitwise_equal(dtype):
    x, w = _inputs(257, 2048, 16384, dtype, 91_000)
    full = gated_linear_batch_invariant(x, w)
    alone = gated_linear_batch_invariant(x[:1], w)
    assert torch.equal(alone, full[:1])


def test_gated_linear_leading_dims_and_fp32_path():
    x, w = _inputs(2 * 50, 256, 512, torch.bfloat16, 92_000)
    x3 = x.view(2, 50, 256)
    out = gated_linear_batch_invariant(x3, w)
    assert out.shape == (2, 50, 512)
    assert torch.equal(out.view(100, 512), gated_linear_batch_invariant(x, w))
    x32, w32 = x.float(), w.float()
    out32 = gated_linear_batch_invariant(x32, w32, "silu")
    assert torch.equal(out32, _composed(x32, w32, "silu"))


def test_gated_linear_rejects_bad_arguments():
    x, w = _inputs(4, 64, 32, torch.bfloat16, 93_000)
    with pytest.raises(ValueError):
        gated_linear_batch_invariant(x, w, "relu")
    with pytest.raises(AssertionError):
        gated_linear_batch_invariant(x, w[:63])
    with pytest.raises(AssertionError):
        gated_linear_batch_invariant(x[:, :32], w)
