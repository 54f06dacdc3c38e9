"""Parity at the benchmark configurations' own shapes.

Config 2 (bf16 linear/addmm sweep, K = 4096, N in {4096, 11008, 16384}, M up
to 8192), config 3 (bf16 attention: 16 query / 4 KV heads, head dim 128,
S in {256, 1024, 4096}, full, top-left causal and a random boolean mask with
P(masked) = 0.1; varlen packing of 32 sequences with lengths U[16, 2048],
TopLeft and BottomRight, Lkv = Lq and Lkv = Lq + delta) and config 4 (bf16
MoE: 8 experts, top-2, hidden 2048, SwiGLU 5632, T in {1, 64, 1024, 4096}).

Every case is checked against the fp64 oracle (oracle/bio_oracle.py) on a
seeded sample of rows / query positions / tokens, so the CPU side stays at a
few seconds per case, with the bf16 bar of the benchmark contract:
normwise relative error <= 1e-2 against fp64, plus the reference suite's
elementwise bf16 tolerance (test_batch_invariance.py:28-32).  Batch
invariance (B = 1 against the first sample of B = N) is checked bitwise at
the same shapes.  Cases mirror test_batch_invariance.py:529-574 (SDPA
causal / mask / GQA), :596-659 (varlen) and :745-766 (MoE).
"""

from __future__ import annotations

import ctypes
import itertools

import pytest
import torch

from batch_invariant_ops import (
    _lib,
    deterministic_token_choice_moe,
    linear_batch_invariant,
    scaled_dot_product_attention_batch_invariant,
    varlen_scaled_dot_product_attention_batch_invariant,
)
from batch_invariant_ops.batch_invariant_ops import addmm_batch_invariant
from conftest import TOLERANCES
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16
NORMWISE_BF16 = 1e-2  # north-star bar for bf16 against the fp64 oracle


def _normwise(out: torch.Tensor, ref: torch.Tensor) -> float:
    out64 = out.double().cpu()
    return float((out64 - ref).norm() / ref.norm().clamp_min(1e-300))


def _check(out: torch.Tensor, ref: torch.Tensor, what: str, scaled_atol: bool = False) -> None:
    """Normwise bar, then elementwise: the reference suite's bf16 tolerance,
    or (scaled_atol) the same rtol with atol taken relative to the largest
    output -- for results built by a chain of bf16 roundings at the scale of
    the whole output (the MoE's rounded routes and partial sums), where one
    element that cancels to a small value keeps the absolute error of its
    large terms."""
    err = _normwise(out, ref)
    assert err <= NORMWISE_BF16, f"{what}: normwise error {err:.3e} > {NORMWISE_BF16}"
    tol = dict(TOLERANCES[BF16])
    if scaled_atol:
        tol["atol"] = tol["atol"] * float(ref.abs().max())
    torch.testing.assert_close(out.double().cpu(), ref, **tol)


def _sample(n: int, count: int, seed: int) -> torch.Tensor:
    """Sorted sample of `count` indices in [0, n): first, last, block edges and
    seeded random positions."""
    fixed = {0, n - 1, min(127, n - 1), min(128, n - 1), n // 2}
    g = torch.Generator().manual_seed(seed)
    rand = torch.randint(0, n, (max(count - len(fixed), 0),), generator=g).tolist()
    return torch.tensor(sorted(fixed | set(rand)), dtype=torch.long)


# --------------------------------------------------------------- config 2
@pytest.mark.parametrize("n", (4096, 11008, 16384))
@pytest.mark.parametrize("layout", ("linear", "addmm"))
def test_config2_full_size_rows_match_oracle(n, layout):
    k, m = 4096, 8192
    gen = torch.Generator(device="cuda").manual_seed(20_000 + n)
    x = torch.randn(m, k, device="cuda", generator=gen).to(BF16)
    w = (torch.randn(n, k, device="cuda", generator=gen) / 64).to(BF16)
    b = (torch.randn(n, device="cuda", generator=gen) * 0.02).to(BF16)
    if layout == "linear":
        run = lambda rows: linear_batch_invariant(rows, w, b)  # noqa: E731
    else:
        w_kn = w.t().contiguous()  # addmm takes W [K, N] row-major
        run = lambda rows: addmm_batch_invariant(b, rows, w_kn)  # noqa: E731
    full = run(x)
    rows = _sample(m, 24, n)
    ref = O.linear(x[rows], w, b)
    _check(full[rows], ref, f"config 2 {layout} N={n} M={m}")
    # B=1 .. B=N: the first row alone and every sweep M give the same bits
    for mm in (1, 8, 32, 128, 512, 2048):
        part = run(x[:mm])
        assert torch.equal(part, full[:mm]), f"M={mm} rows differ from the M={m} run"


# --------------------------------------------------------------- config 3
def _attn_inputs(batch, seq, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, 16, seq, 128, device="cuda", generator=gen).to(BF16)
    k = torch.randn(batch, 4, seq, 128, device="cuda", generator=gen).to(BF16)
    v = torch.randn(batch, 4, seq, 128, device="cuda", generator=gen).to(BF16)
    keep = torch.rand(batch, 1, seq, seq, device="cuda", generator=gen) > 0.1
    return q, k, v, keep


@pytest.mark.parametrize("seq", (256, 1024, 4096))
@pytest.mark.parametrize("mode", ("full", "causal", "mask"))
def test_config3_sdpa_gqa_d128_matches_oracle(seq, mode):
    q, k, v, keep = _attn_inputs(2, seq, 30_000 + seq)
    mask = keep if mode == "mask" else None
    out = scaled_dot_product_attention_batch_invariant(
        q, k, v, attn_mask=mask, is_causal=mode == "causal", enable_gqa=True)
    rows = _sample(seq, 40, seq)
    ref = O.sdpa(q, k, v, attn_mask=mask, is_causal=mode == "causal", enable_gqa=True,
                 query_rows=rows)
    _check(out[:, :, rows], ref, f"sdpa S={seq} {mode}")
    alone = scaled_dot_product_attention_batch_invariant(
        q[:1], k[:1], v[:1], attn_mask=None if mask is None else mask[:1],
        is_causal=mode == "causal", enable_gqa=True)
    assert torch.equal(alone, out[:1]), f"sdpa S={seq} {mode}: B=1 differs from B=2"


@pytest.mark.parametrize("mode", ("full", "causal", "mask"))
def test_config3_sdpa_batch_eight_first_sample_bitwise(mode):
    q, k, v, keep = _attn_inputs(8, 1024, 31_000)
    mask = keep if mode == "mask" else None
    out = scaled_dot_product_attention_batch_invariant(
        q, k, v, attn_mask=mask, is_causal=mode == "causal", enable_gqa=True)
    for b in (1, 3):
        part = scaled_dot_product_attention_batch_invariant(
            q[:b], k[:b], v[:b], attn_mask=None if mask is None else mask[:b],
            is_causal=mode == "causal", enable_gqa=True)
        assert torch.equal(part, out[:b])


def _varlen_lengths(seed):
    g = torch.Generator().manual_seed(seed)
    lq = torch.randint(16, 2049, (32,), generator=g).tolist()
    delta = torch.randint(1, 65, (32,), generator=g).tolist()
    return lq, delta


def _cu(lengths):
    return torch.tensor([0, *itertools.accumulate(lengths)], device="cuda", dtype=torch.int32)


@pytest.mark.parametrize("causal_type", ("TopLeft", "BottomRight"))
@pytest.mark.parametrize("kv_longer", (False, True))
def test_config3_varlen_32_sequences_matches_oracle(causal_type, kv_longer):
    lq, delta = _varlen_lengths(32_000)
    lk = [a + d for a, d in zip(lq, delta)] if kv_longer else list(lq)
    gen = torch.Generator(device="cuda").manual_seed(32_001)
    q = torch.randn(1, sum(lq), 16, 128, device="cuda", generator=gen).to(BF16)
    k = torch.randn(1, sum(lk), 4, 128, device="cuda", generator=gen).to(BF16)
    v = torch.randn(1, sum(lk), 4, 128, device="cuda", generator=gen).to(BF16)
    cu_q, cu_k = _cu(lq), _cu(lk)
    out = varlen_scaled_dot_product_attention_batch_invariant(
        q, k, v, cu_q, cu_k, is_causal=True, causal_type=causal_type)
    # per sequence: first, last and three seeded positions
    g = torch.Generator().manual_seed(32_002)
    tokens, start = [], 0
    for n in lq:
        picks = {0, n - 1, *torch.randint(0, n, (3,), generator=g).tolist()}
        tokens += [start + p for p in sorted(picks)]
        start += n
    ref = O.varlen_sdpa(q, k, v, cu_q, cu_k, True, causal_type, query_tokens=tokens)
    idx = torch.tensor(tokens)
    _check(out[:, idx], ref[:, idx], f"varlen {causal_type} kv_longer={kv_longer}")
    # one sequence packed alone gives the bits it gets inside the pack
    s = 5
    qs, qe, ks, ke = sum(lq[:s]), sum(lq[: s + 1]), sum(lk[:s]), sum(lk[: s + 1])
    alone = varlen_scaled_dot_product_attention_batch_invariant(
        q[:, qs:qe].contiguous(), k[:, ks:ke].contiguous(), v[:, ks:ke].contiguous(),
        _cu([lq[s]]), _cu([lk[s]]), is_causal=True, causal_type=causal_type)
    assert torch.equal(alone, out[:, qs:qe])


# --------------------------------------------------------------- config 4
_MOE_WEIGHTS: dict = {}


def _moe_weights():
    if not _MOE_WEIGHTS:
        gen = torch.Generator(device="cuda").manual_seed(40_000)
        _MOE_WEIGHTS["gate"] = (torch.randn(8, 5632, 2048, device="cuda", generator=gen) * 0.02).to(BF16)
        _MOE_WEIGHTS["up"] = (torch.randn(8, 5632, 2048, device="cuda", generator=gen) * 0.02).to(BF16)
        _MOE_WEIGHTS["down"] = (torch.randn(8, 2048, 5632, device="cuda", generator=gen) * 0.02).to(BF16)
    return _MOE_WEIGHTS["gate"], _MOE_WEIGHTS["up"], _MOE_WEIGHTS["down"]


def _route(tokens, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    hidden = torch.randn(tokens, 2048, device="cuda", generator=gen).to(BF16)
    logits = torch.randn(tokens, 8, device="cuda", generator=gen)  # fp32 router logits
    top, sel = torch.topk(logits, 2)
    return hidden, torch.softmax(top, -1), sel, logits


@pytest.mark.parametrize("tokens", (1, 64, 1024, 4096))
def test_config4_moe_matches_oracle(tokens):
    gate, up, down = _moe_weights()
    hidden, weights, sel, logits = _route(tokens, 41_000 + tokens)
    out = deterministic_token_choice_moe(hidden, weights, sel, gate, up, down)
    picks = _sample(tokens, 48, tokens) if tokens > 48 else torch.arange(tokens)
    ref = O.moe(hidden[picks], weights[picks], sel[picks], gate, up, down)
    _check(out[picks], ref, f"moe T={tokens}", scaled_atol=True)
    # the route plan (integer work) equals the oracle's stable sort bit for bit
    lib = _lib.load()
    s = tokens * 2
    nbytes = lib.bio_moe_plan_workspace(8, tokens, 2)
    ws = torch.full((nbytes // 4,), -7, dtype=torch.int32, device="cuda")
    _lib.check(lib.bio_moe_plan(ctypes.c_void_p(sel.data_ptr()), 8, tokens, 2,
                                ctypes.c_void_p(ws.data_ptr()), nbytes, 0, _lib.stream_of(sel)),
               "bio_moe_plan")
    e_seg, e_slot, e_tok = O.moe_route_plan(sel, 8)
    got = ws.cpu().long()
    assert torch.equal(got[:9], e_seg)
    assert torch.equal(got[9 : 9 + s], e_slot)
    assert torch.equal(got[9 + s : 9 + 2 * s][: int(e_seg[-1])], e_tok)
    # the selected experts are the top-2 logits with the lowest-index
    # tie-break of the oracle's router (fp32 logits: no ties expected)
    o_w, o_sel = O.topk_routing(logits, 2)
    assert torch.equal(o_sel, sel.cpu().long())
    # batch invariance: the first token alone, and the first 7 tokens
    for t in (1, min(7, tokens)):
        part = deterministic_token_choice_moe(hidden[:t], weights[:t], sel[:t], gate, up, down)
        assert torch.equal(part, out[:t]), f"moe T={tokens}: first {t} tokens differ"
