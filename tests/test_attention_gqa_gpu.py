"""Grouped-query packing of the one-tile attention kernel.

When several query heads share a KV head (group of 2, 4, 8 or 16) and the
one-tile kernel runs, the heads of a group fill one 128-row tile together
(128 / group tokens each).  A row's arithmetic depends only on its query row,
its KV head's keys/values and the fixed key blocks, so the packed result must
equal, bit for bit, the same attention run with the KV heads repeated (no
grouping, hence no packing) -- and stay within the bf16/fp16 bar of the fp64
oracle.  Shapes include the VLA action expert (8 query heads on one KV head,
50 queries over 354 keys, head dim 256), short decode-like queries, causal
masks (top-left), boolean
and additive masks, and head dims that are padded.
"""

from __future__ import annotations

import pytest
import torch

from batch_invariant_ops import scaled_dot_product_attention_batch_invariant as sdpa
from conftest import DTYPES
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
HALF = tuple(d for d in DTYPES if d != torch.float32)

CASES = [
    # (batch, heads, kv_heads, lq, lk, d)
    (3, 8, 1, 50, 354, 256),    # VLA action expert
    (2, 8, 1, 304, 304, 256),   # VLA prefix LM
    (2, 16, 4, 77, 200, 128),   # group 4, one-tile (lq <= 128)
    (2, 4, 2, 5, 33, 64),       # group 2, decode-like
    (1, 32, 2, 1, 129, 96),     # group 16, one token, padded head dim
    (2, 8, 1, 19, 70, 200),     # padded head dim 200 -> 256
]


def _qkv(b, h, hk, lq, lk, d, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(b, lq, h, d, device="cuda", generator=g).to(dtype).transpose(1, 2)
    k = torch.randn(b, lk, hk, d, device="cuda", generator=g).to(dtype).transpose(1, 2)
    v = torch.randn(b, lk, hk, d, device="cuda", generator=g).to(dtype).transpose(1, 2)
    return q, k, v


def _repeat(t, group):
    return t.repeat_interleave(group, dim=1)


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("causal", (False, True))
def test_packed_gqa_equals_repeated_heads_and_oracle(dtype, case, causal):
    b, h, hk, lq, lk, d = case
    q, k, v = _qkv(b, h, hk, lq, lk, d, dtype, 5_000 + lq + d)
    packed = sdpa(q, k, v, is_causal=causal, enable_gqa=True)
    plain = sdpa(q, _repeat(k, h // hk), _repeat(v, h // hk), is_causal=causal)
    assert torch.equal(packed, plain)
    rows = torch.arange(0, lq, max(1, lq // 8))
    ref = O.sdpa(q, k, v, is_causal=causal, enable_gqa=True, query_rows=rows)
    out = packed[:, :, rows].double().cpu()
    err = float((out - ref).norm() / ref.norm().clamp_min(1e-30))
    assert err <= 1e-2, err


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("kind", ("bool", "additive"))
def test_packed_gqa_with_masks(dtype, kind):
    b, h, hk, lq, lk, d = 2, 8, 2, 40, 150, 256
    q, k, v = _qkv(b, h, hk, lq, lk, d, dtype, 6_000)
    g = torch.Generator(device="cuda").manual_seed(6_001)
    if kind == "bool":
        mask = torch.rand(b, h, lq, lk, device="cuda", generator=g) > 0.1
    else:
        mask = (torch.randn(b, 1, lq, lk, device="cuda", generator=g) * 2).to(dtype)
    packed = sdpa(q, k, v, attn_mask=mask, enable_gqa=True)
    plain = sdpa(q, _repeat(k, h // hk), _repeat(v, h // hk), attn_mask=mask)
    assert torch.equal(packed, plain)
    ref = O.sdpa(q, k, v, attn_mask=mask, enable_gqa=True)
    err = float((packed.double().cpu() - ref).norm() / ref.norm())
    assert err <= 1e-2, err


@pytest.mark.parametrize("dtype", HALF)
def test_packed_gqa_first_sample_alone_is_bitwise_equal(dtype):
    q, k, v = _qkv(5, 8, 1, 50, 354, 256, dtype, 7_000)
    full = sdpa(q, k, v, enable_gqa=True)
    alone = sdpa(q[:1], k[:1], v[:1], enable_gqa=True)
    assert torch.equal(alone, full[:1])
