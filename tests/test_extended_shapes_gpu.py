"""Extended shape regression suite: every operator shape the
reference benchmarked on real VLA models (tests/golden/extended_shapes.json,
extracted from its research/*/benchmarks.json by make_extended_shapes.py) --
LM heads up to 184,622 wide, Cosmos varlen attention over ~3.1k-token
sequences, the LingBot fp32 32-expert top-4 MoE, Qwen depthwise conv1d,
ZoeDepth/UVA transposed convolutions, SigLIP/Florence patch convolutions.

Each case runs once on the full benchmarked batch and once on its first
sample (first sequence for varlen, first robot's tokens for the MoE); the
first sample's outputs must match bit for bit, and the full output must match
an fp64 computation normwise (bf16/fp16 1e-2, fp32 1e-5)."""

from __future__ import annotations

import json
import zlib
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

import batch_invariant_ops as bio
from batch_invariant_ops.batch_invariant_ops import (
    addmm_batch_invariant,
    bmm_batch_invariant,
    mm_batch_invariant,
)

pytestmark = pytest.mark.gpu
CASES = json.loads((Path(__file__).resolve().parent / "golden" / "extended_shapes.json")
                   .read_text())["cases"]
DT = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16,
      "torch.float32": torch.float32}


def _rand(shape, dtype, gen, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=gen) * scale).to(dtype)


def _close(out, ref, dtype):
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    err = float((out.double() - ref).norm() / ref.norm().clamp_min(1e-30))
    assert err <= tol, err


def _batch(x, gen, n=3):
    """x with its leading dimension grown to at least n by random companions."""
    if x.shape[0] >= n:
        return x
    extra = _rand((n - x.shape[0], *x.shape[1:]), x.dtype, gen)
    return torch.cat([x, extra])


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_extended_shape(case):
    kind, sh = case["kind"], case["shape"]
    dtype = DT[sh["dtype"]]
    gen = torch.Generator(device="cuda").manual_seed(zlib.crc32(case["id"].encode()))
    if kind in ("mm", "addmm"):
        left = _batch(_rand(sh["left"], dtype, gen), gen)
        right = _rand(sh["right"], dtype, gen, scale=sh["right"][0] ** -0.5)
        if left.ndim == 3:  # batched products (attention bmm, per-expert weights)
            right = _batch(right, gen)[: left.shape[0]]
            full = bmm_batch_invariant(left, right)
            one = bmm_batch_invariant(left[:1], right[:1])
            assert torch.equal(one, full[:1])
            _close(full, torch.bmm(left.double(), right.double()), dtype)
            return
        if kind == "addmm":
            bias = _rand(sh["bias"], dtype, gen, scale=0.1)
            full = addmm_batch_invariant(bias, left, right)
            one = addmm_batch_invariant(bias, left[:1], right)
            ref = left.double() @ right.double() + bias.double()
        else:
            full = mm_batch_invariant(left, right)
            one = mm_batch_invariant(left[:1], right)
            ref = left.double() @ right.double()
        assert torch.equal(one, full[:1])
        _close(full, ref, dtype)
    elif kind == "linear":
        x = _batch(_rand(sh["input"], dtype, gen), gen)
        w = _rand(sh["weight"], dtype, gen, scale=sh["weight"][1] ** -0.5)
        b = _rand(sh["bias"], dtype, gen, scale=0.1) if sh.get("bias") else None
        full = bio.linear_batch_invariant(x, w, b)
        assert torch.equal(bio.linear_batch_invariant(x[:1], w, b), full[:1])
        ref = x.double() @ w.double().t() + (b.double() if b is not None else 0)
        _close(full, ref, dtype)
    elif kind == "sdpa":
        q = _batch(_rand(sh["query"], dtype, gen), gen)
        k = _batch(_rand(sh["key"], dtype, gen), gen)[: q.shape[0]]
        v = _batch(_rand(sh["value"], dtype, gen), gen)[: q.shape[0]]
        gqa = q.shape[1] != k.shape[1]
        causal = bool(sh["causal"])
        full = bio.scaled_dot_product_attention_batch_invariant(q, k, v, is_causal=causal,
                                                                 enable_gqa=gqa)
        one = bio.scaled_dot_product_attention_batch_invariant(q[:1], k[:1], v[:1],
                                                                is_causal=causal, enable_gqa=gqa)
        assert torch.equal(one, full[:1])
        ref = F.scaled_dot_product_attention(q[:1].float(), k[:1].float(), v[:1].float(),
                                             is_causal=causal, enable_gqa=gqa)
        _close(one, ref.double(), dtype)
    elif kind == "varlen":
        lq, lk = sh["logical_query_length"], sh["logical_kv_length"]
        nseq = max(2, sh["query"][1] // lq)
        hq, hk, d = sh["query_heads"], sh["kv_heads"], sh["head_dim"]
        q = _rand((1, nseq * lq, hq, d), dtype, gen)
        k = _rand((1, nseq * lk, hk, d), dtype, gen)
        v = _rand((1, nseq * lk, hk, d), dtype, gen)
        cq = torch.arange(nseq + 1, device="cuda", dtype=torch.int32) * lq
        ck = torch.arange(nseq + 1, device="cuda", dtype=torch.int32) * lk
        causal = bool(sh["causal"])
        full = bio.varlen_scaled_dot_product_attention_batch_invariant(q, k, v, cq, ck,
                                                                      is_causal=causal)
        one = bio.varlen_scaled_dot_product_attention_batch_invariant(
            q[:, :lq], k[:, :lk], v[:, :lk], cq[:2], ck[:2], is_causal=causal)
        assert torch.equal(one, full[:, :lq])
        ref = F.scaled_dot_product_attention(
            q[:, :lq].transpose(1, 2).float(), k[:, :lk].transpose(1, 2).float(),
            v[:, :lk].transpose(1, 2).float(), is_causal=causal, enable_gqa=True)
        _close(one, ref.transpose(1, 2).double(), dtype)
    elif kind in ("conv", "depthwise_conv1d", "conv_transpose"):
        x = _batch(_rand(sh["input"], dtype, gen), gen)
        w = _rand(sh["weight"], dtype, gen, scale=0.05)
        b = _rand(sh["bias"], dtype, gen, scale=0.1) if sh.get("bias") else None
        nd = x.ndim - 2
        stride = tuple(sh.get("stride", [1] * nd))
        padding = tuple(sh.get("padding", [0] * nd))
        groups = int(sh.get("groups", 1))
        if kind == "conv_transpose":
            fn = {2: bio.conv_transpose2d_batch_invariant, 3: bio.conv_transpose3d_batch_invariant}[nd]
            run = lambda t: fn(t, w, b, stride, padding, (1,) * nd, (0,) * nd, groups)  # noqa: E731
            tfn = {2: F.conv_transpose2d, 3: F.conv_transpose3d}[nd]
            ref = tfn(x.double(), w.double(), b.double() if b is not None else None,
                      stride=stride, padding=padding, groups=groups)
        else:
            fn = {1: bio.conv1d_batch_invariant, 2: bio.conv2d_batch_invariant,
                  3: bio.conv3d_batch_invariant}[nd]
            run = lambda t: fn(t, w, b, stride, padding, (1,) * nd, False, (0,) * nd, groups)  # noqa: E731
            tfn = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
            ref = tfn(x.double(), w.double(), b.double() if b is not None else None,
                      stride=stride, padding=padding, groups=groups)
        full = run(x)
        assert torch.equal(run(x[:1]), full[:1])
        _close(full, ref, dtype)
    elif kind == "mean":
        x = _batch(_rand(sh["input"], dtype, gen), gen)
        dim = sh.get("dimension", sh.get("dim"))
        keep = bool(sh.get("keepdim", False))
        full = bio.mean_dim(x, dim, keep)
        assert torch.equal(bio.mean_dim(x[:1], dim, keep), full[:1])
        _close(full, x.double().mean(dim, keepdim=keep), dtype)
    elif kind == "vector_norm":
        x = _batch(_rand(sh["input"], dtype, gen), gen)
        full = bio.linalg_vector_norm_batch_invariant(x, dim=sh["dim"])
        assert torch.equal(bio.linalg_vector_norm_batch_invariant(x[:1], dim=sh["dim"]), full[:1])
        _close(full, torch.linalg.vector_norm(x.double(), dim=sh["dim"]), dtype)
    elif kind == "moe":
        t, dmodel = sh["hidden"]
        e, k, inter = sh["experts"], sh["top_k"], sh["intermediate"]
        robots = max(1, int(sh.get("logical_robot_batch", 1)))
        per = t // robots
        hid = _rand((t, dmodel), dtype, gen)
        gate = _rand((e, inter, dmodel), dtype, gen, scale=0.02)
        up = _rand((e, inter, dmodel), dtype, gen, scale=0.02)
        down = _rand((e, dmodel, inter), dtype, gen, scale=0.02)
        logits = torch.randn(t, e, device="cuda", generator=gen)
        top, sel = torch.topk(logits, k)
        rw = torch.softmax(top, -1).to(dtype)
        full = bio.deterministic_token_choice_moe(hid, rw, sel, gate, up, down)
        one = bio.deterministic_token_choice_moe(hid[:per], rw[:per], sel[:per], gate, up, down)
        assert torch.equal(one, full[:per])
        ref = torch.zeros(t, dmodel, dtype=torch.float64, device="cuda")
        h64 = hid.double()
        for j in range(k):
            ex = sel[:, j]
            g = torch.einsum("td,tid->ti", h64, gate.double()[ex])
            u = torch.einsum("td,tid->ti", h64, up.double()[ex])
            y = torch.einsum("ti,tdi->td", F.silu(g) * u, down.double()[ex])
            ref += rw[:, j].double()[:, None] * y
        _close(full, ref, dtype)
    else:  # pragma: no cover - the extractor only emits the kinds above
        pytest.fail(f"unknown kind {kind}")


def test_every_case_kind_is_covered():
    kinds = {c["kind"] for c in CASES}
    assert kinds == {"mm", "addmm", "linear", "sdpa", "varlen", "conv", "depthwise_conv1d",
                     "conv_transpose", "mean", "vector_norm", "moe"}
    assert any(c["shape"].get("right", [0, 0])[1] == 184622 for c in CASES)  # UniVLA LM head
    assert any(c["kind"] == "moe" and c["shape"]["experts"] == 32 for c in CASES)

