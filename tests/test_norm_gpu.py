"""Fused batch-invariant LayerNorm / RMSNorm (bio_norm).

Checked against the fp64 oracle at the VLA model's widths (1152 vision,
2048 prefix LM, 1024 action expert) and at the kernel family's switch
points (warp per row up to 2048, one 256-thread CTA per row up to 16384,
a 1024-thread loop beyond, ragged widths that are not multiples of 8);
bitwise for B=1 against the first row of B=N, and for a row read from an
unaligned view against the same row read aligned; and through the mode, where
F.layer_norm / F.rms_norm must reach these kernels.  The reference builds
RMSNorm from mean_dim and tests it through F.normalize
(test_batch_invariance.py:492-509).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from batch_invariant_ops import (
    layer_norm_batch_invariant,
    rms_norm_batch_invariant,
    set_batch_invariant_mode,
)
from batch_invariant_ops.batch_invariant_ops import native_layer_norm_batch_invariant
from conftest import DTYPES, TOLERANCES
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
WIDTHS = (64, 200, 1024, 1152, 2048, 2056, 4096, 5000, 16384, 20000)


def _inputs(rows, n, dtype, seed, affine=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(rows, n, device="cuda", generator=g) * 2 + 0.5).to(dtype)
    w = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).to(dtype) if affine else None
    b = (0.1 * torch.randn(n, device="cuda", generator=g)).to(dtype) if affine else None
    return x, w, b


def _normwise(out, ref):
    return float((out.double().cpu() - ref).norm() / ref.norm())


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", WIDTHS)
@pytest.mark.parametrize("rms", (False, True))
def test_norm_matches_oracle_and_is_batch_invariant(dtype, n, rms):
    x, w, b = _inputs(37, n, dtype, 70_000 + n)
    if rms:
        out = rms_norm_batch_invariant(x, (n,), w, eps=1e-6)
        ref = O.rms_norm(x, 1, w, eps=1e-6)
        alone = rms_norm_batch_invariant(x[:1], (n,), w, eps=1e-6)
    else:
        out = layer_norm_batch_invariant(x, (n,), w, b, eps=1e-5)
        ref = O.layer_norm(x, 1, w, b, eps=1e-5)
        alone = layer_norm_batch_invariant(x[:1], (n,), w, b, eps=1e-5)
    bar = 1e-5 if dtype == torch.float32 else 1e-2
    assert _normwise(out, ref) <= bar
    torch.testing.assert_close(out.double().cpu(), ref, **TOLERANCES[dtype])
    assert torch.equal(alone, out[:1])


@pytest.mark.parametrize("n", (1152, 2048, 5000))
def test_unaligned_rows_give_the_aligned_bits(n):
    # the vector and element load paths run the same sums in the same order
    x, w, b = _inputs(9, n + 1, torch.bfloat16, 71_000 + n)
    base = layer_norm_batch_invariant(x[:, 1:].contiguous(), (n,), w[1:], b[1:])
    flat = x[:, 1:].contiguous().reshape(-1)
    shifted = torch.empty(flat.numel() + 1, device="cuda", dtype=flat.dtype)
    shifted[1:] = flat
    view = shifted[1:].view(9, n)  # data pointer 2 bytes past a 16-byte boundary
    out = layer_norm_batch_invariant(view, (n,), w[1:], b[1:])
    assert torch.equal(out, base)


def test_native_layer_norm_statistics_and_mode_routing():
    x, w, b = _inputs(3 * 5, 1152, torch.bfloat16, 72_000)
    x = x.view(3, 5, 1152)
    out, mean, rstd = native_layer_norm_batch_invariant(x, [1152], w, b, 1e-6)
    assert mean.shape == (3, 5, 1) and rstd.shape == (3, 5, 1) and mean.dtype == torch.float32
    x64 = x.double().cpu()
    torch.testing.assert_close(mean.double().cpu(), x64.mean(-1, keepdim=True), rtol=1e-5,
                               atol=1e-5)
    var = x64.var(-1, unbiased=False, keepdim=True)
    torch.testing.assert_close(rstd.double().cpu(), 1 / torch.sqrt(var + 1e-6), rtol=1e-4,
                               atol=1e-5)
    mine = layer_norm_batch_invariant(x, (1152,), w, b, 1e-6)
    mine_rms = rms_norm_batch_invariant(x, (1152,), w, 1e-6)
    with torch.inference_mode(), set_batch_invariant_mode():
        via_mode = F.layer_norm(x, (1152,), w, b, 1e-6)
        via_mode_rms = F.rms_norm(x, (1152,), w, 1e-6)
    assert torch.equal(via_mode, mine)
    assert torch.equal(via_mode_rms, mine_rms)


def test_norm_without_affine_and_empty():
    x, _, _ = _inputs(4, 1024, torch.float16, 73_000, affine=False)
    torch.testing.assert_close(layer_norm_batch_invariant(x, (1024,)).double().cpu(),
                               O.layer_norm(x, 1), **TOLERANCES[torch.float16])
    torch.testing.assert_close(rms_norm_batch_invariant(x, (1024,)).double().cpu(),
                               O.rms_norm(x, 1), **TOLERANCES[torch.float16])
    empty = torch.empty(0, 1024, device="cuda", dtype=torch.bfloat16)
    assert layer_norm_batch_invariant(empty, (1024,)).shape == (0, 1024)
