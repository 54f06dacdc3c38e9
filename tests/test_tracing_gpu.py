"""Per-launch records (the counterpart of the reference's Triton launch
metadata, batch_invariant_ops.py:31-47: a name carrying the problem sizes
plus the algorithmic flops and bytes of each matmul launch)."""

from __future__ import annotations

import pytest
import torch

import batch_invariant_ops as bio
from batch_invariant_ops import tracing

pytestmark = pytest.mark.gpu


def test_records_name_flops_and_bytes_of_each_call():
    g = torch.Generator(device="cuda").manual_seed(80_000)
    x = torch.randn(37, 512, device="cuda", generator=g).bfloat16()
    w = torch.randn(256, 512, device="cuda", generator=g).bfloat16()
    q = torch.randn(2, 4, 64, 64, device="cuda", generator=g).bfloat16()
    with tracing.record_launches(nvtx=True) as rec:
        bio.linear_batch_invariant(x, w)
        bio.scaled_dot_product_attention_batch_invariant(q, q, q, is_causal=True)
        bio.softmax(x, -1)
        bio.layer_norm_batch_invariant(x, (512,))
    ops = [r["op"] for r in rec]
    assert ops == ["gemm", "attention", "softmax", "norm"], ops
    gemm = rec[0]
    assert gemm["name"] == "bio_gemm [M=37, N=256, K=512, batch=1]"
    assert gemm["flops16"] == 2.0 * 37 * 256 * 512
    assert gemm["bytes"] == 2 * (37 * 512 + 512 * 256 + 37 * 256)
    assert rec[1]["flops16"] == 2.0 * 2 * 4 * 64 * 64 * 128 / 2
    assert rec[2]["bytes"] == 2 * 2 * x.numel()
    # nothing is recorded outside the context
    bio.linear_batch_invariant(x, w)
    assert len(rec) == 4
