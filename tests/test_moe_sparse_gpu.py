"""Sparse MoE path: the route plan (bit-exact against the oracle's stable
sort), the segmented expert GEMM (each segment's rows bit-identical to a
plain GEMM of those rows) and the whole sparse MoE (bit-identical to the
dense all-experts evaluation of the reference's schedule, moe.py:67-92)."""

from __future__ import annotations

import ctypes

import pytest
import torch

from batch_invariant_ops import _gemm, _lib, deterministic_token_choice_moe
from batch_invariant_ops import moe as moe_mod
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
HALF = (torch.float16, torch.bfloat16)


def _rn(*shape, dtype, gen, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=gen) * scale).to(dtype)


def _plan(sel: torch.Tensor, experts: int) -> torch.Tensor:
    lib = _lib.load()
    tokens, top_k = sel.shape
    nbytes = lib.bio_moe_plan_workspace(experts, tokens, top_k)
    assert nbytes > 0
    ws = torch.full((nbytes // 4,), -7, dtype=torch.int32, device="cuda")
    _lib.check(lib.bio_moe_plan(ctypes.c_void_p(sel.data_ptr()), experts, tokens, top_k,
                                ctypes.c_void_p(ws.data_ptr()), nbytes, 0,
                                _lib.stream_of(sel)), "bio_moe_plan")
    return ws


@pytest.mark.parametrize(
    "tokens,top_k,experts",
    [(1, 1, 1), (5, 2, 3), (37, 4, 7), (1000, 2, 8), (3000, 8, 64), (513, 3, 1024)],
)
def test_route_plan_matches_stable_sort(tokens, top_k, experts):
    gen = torch.Generator(device="cuda").manual_seed(tokens * 31 + experts)
    sel = torch.randint(0, experts, (tokens, top_k), device="cuda", generator=gen)
    ws = _plan(sel, experts)
    seg, slot_row, row_token = O.moe_route_plan(sel, experts)
    s = tokens * top_k
    got = ws.cpu().long()
    assert torch.equal(got[: experts + 1], seg)
    assert torch.equal(got[experts + 1 : experts + 1 + s], slot_row)
    rt = got[experts + 1 + s : experts + 1 + 2 * s]
    assert torch.equal(rt[: int(seg[-1])], row_token)


def test_route_plan_skewed_and_invalid_ids():
    sel = torch.tensor([[2, 2], [2, 0], [9, 2], [-1, 1], [2, 2]], device="cuda")
    _lib.clear_device_status()
    ws = _plan(sel, 3)
    assert _lib.device_status() & _lib.BIO_DEV_INDEX
    _lib.clear_device_status()
    seg, slot_row, _ = O.moe_route_plan(sel, 3)
    got = ws.cpu().long()
    assert torch.equal(got[:4], seg)
    assert torch.equal(got[4 : 4 + 10], slot_row)
    assert int(seg[-1]) == 8 and (slot_row == -1).sum() == 2


def _segmented(x, w, seg_list, out=None):
    seg = torch.tensor(seg_list, dtype=torch.int32, device="cuda")
    e, n, k = w.shape
    rows = x.shape[0]
    y = out if out is not None else torch.empty((rows, n), device="cuda", dtype=x.dtype)
    opa = _gemm.operand_a(x, e, 1, rows, k, x.stride(0), x.stride(1), 0, 0)
    opb = _gemm.operand_b(w, e, 1, k, n, w.stride(2), w.stride(1), w.stride(0), 0)
    _gemm.launch(opa, opb, y, batch1=e, batch2=1, m=rows, n=n, k=k, c_sm=n, c_sn=1, c_s1=0,
                 c_s2=0, segments=seg)
    return y


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize(
    "sizes,n,k",
    [
        ((0, 1, 127, 128, 129, 300), 200, 136),
        ((513, 0, 0, 7), 512, 1000),
        ((40,) * 9, 64, 64),
        ((1,), 5632, 2048),
        ((700, 650, 20), 2048, 512),
    ],
)
def test_segmented_gemm_rows_match_plain_gemm(dtype, sizes, n, k):
    gen = torch.Generator(device="cuda").manual_seed(sum(sizes) + n + k)
    seg = [0]
    for r in sizes:
        seg.append(seg[-1] + r)
    rows = seg[-1] + 3  # three trailing rows outside every segment
    x = _rn(rows, k, dtype=dtype, gen=gen)
    w = _rn(len(sizes), n, k, dtype=dtype, gen=gen, scale=k**-0.5)
    sentinel = torch.full((rows, n), 7.0, device="cuda", dtype=dtype)
    y = _segmented(x, w, seg, out=sentinel)
    for s, (lo, hi) in enumerate(zip(seg[:-1], seg[1:])):
        if hi > lo:
            ref = _gemm.mm(x[lo:hi], w[s].t())
            assert torch.equal(y[lo:hi], ref), s
    assert torch.all(y[seg[-1] :] == 7.0)


def test_segmented_gemm_rejects_bad_arguments_and_flags_bad_offsets():
    x = torch.randn(64, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2, 64, 64, device="cuda", dtype=torch.bfloat16)
    # offsets out of order / beyond m: that segment is skipped and flagged
    _lib.clear_device_status()
    y = torch.zeros(64, 64, device="cuda", dtype=torch.bfloat16)
    _segmented(x, w, [0, 40, 80], out=y)  # segment 1 ends past m = 64
    torch.cuda.synchronize()
    assert _lib.device_status() & _lib.BIO_DEV_INDEX
    _lib.clear_device_status()
    assert torch.equal(y[:40], _gemm.mm(x[:40], w[0].t()))
    assert torch.count_nonzero(y[40:]) == 0
    # fp32 is not a segmented dtype
    x32 = x.float()
    with pytest.raises(RuntimeError):
        _segmented(x32, w.float(), [0, 32, 64])


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize(
    "tokens,experts,top_k,hidden,inter",
    [(1, 4, 1, 64, 80), (11, 7, 4, 64, 80), (257, 8, 2, 256, 512), (1024, 8, 2, 2048, 5632),
     (300, 32, 4, 512, 384), (64, 3, 3, 72, 40)],
)
def test_sparse_moe_equals_dense_bitwise(dtype, tokens, experts, top_k, hidden, inter):
    gen = torch.Generator(device="cuda").manual_seed(tokens + 13 * experts + hidden)
    h = _rn(tokens, hidden, dtype=dtype, gen=gen)
    gate = _rn(experts, inter, hidden, dtype=dtype, gen=gen, scale=hidden**-0.5)
    up = _rn(experts, inter, hidden, dtype=dtype, gen=gen, scale=hidden**-0.5)
    down = _rn(experts, hidden, inter, dtype=dtype, gen=gen, scale=inter**-0.5)
    logits = torch.randn(tokens, experts, device="cuda", generator=gen)
    top, sel = torch.topk(logits, top_k)
    w = torch.softmax(top, -1).to(dtype)
    assert moe_mod.sparse_path_applies(dtype, experts, tokens, top_k, inter, hidden)
    sparse = deterministic_token_choice_moe(h, w, sel, gate, up, down)
    dense = moe_mod._dense_moe(h, w, sel.long().contiguous(), gate, up, down)
    assert torch.equal(sparse, dense)
    alone = deterministic_token_choice_moe(h[:1], w[:1], sel[:1], gate, up, down)
    assert torch.equal(alone, sparse[:1])


@pytest.mark.parametrize("dtype", HALF)
def test_sparse_moe_skewed_routing_and_repeated_experts(dtype):
    """Every token on the same expert (one large segment, the others empty),
    and a token that picks one expert twice."""
    gen = torch.Generator(device="cuda").manual_seed(99)
    tokens, experts, hidden, inter = 600, 5, 128, 96
    h = _rn(tokens, hidden, dtype=dtype, gen=gen)
    gate = _rn(experts, inter, hidden, dtype=dtype, gen=gen, scale=0.1)
    up = _rn(experts, inter, hidden, dtype=dtype, gen=gen, scale=0.1)
    down = _rn(experts, hidden, inter, dtype=dtype, gen=gen, scale=0.1)
    sel = torch.full((tokens, 2), 3, device="cuda", dtype=torch.int64)
    sel[5, 1] = 0
    w = torch.rand(tokens, 2, device="cuda", generator=gen).to(dtype)
    sparse = deterministic_token_choice_moe(h, w, sel, gate, up, down)
    dense = moe_mod._dense_moe(h, w, sel, gate, up, down)
    assert torch.equal(sparse, dense)


def test_sparse_moe_out_of_range_expert_zeroes_row():
    gen = torch.Generator(device="cuda").manual_seed(5)
    h = _rn(3, 16, dtype=torch.bfloat16, gen=gen)
    gate = _rn(2, 8, 16, dtype=torch.bfloat16, gen=gen)
    down = _rn(2, 16, 8, dtype=torch.bfloat16, gen=gen)
    sel = torch.tensor([[0, 1], [1, 5], [0, 0]], device="cuda")
    w = torch.rand(3, 2, device="cuda", generator=gen)
    _lib.clear_device_status()
    out = deterministic_token_choice_moe(h, w, sel, gate, gate, down)
    assert _lib.device_status() & _lib.BIO_DEV_INDEX
    _lib.clear_device_status()
    assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[0]) > 0
    dense = moe_mod._dense_moe(h, w, sel, gate, gate, down)
    _lib.clear_device_status()
    assert torch.equal(out, dense)


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("t,e,n,k", [(1, 2, 80, 64), (37, 3, 200, 136), (300, 4, 5632, 512),
                                     (129, 2, 128, 2048), (1024, 1, 384, 1000)])
def test_fused_swiglu_gemm_equals_separate_gemms_and_silu(dtype, t, e, n, k):
    gen = torch.Generator(device="cuda").manual_seed(t * 7 + n + k)
    x = _rn(t, k, dtype=dtype, gen=gen)
    gate = _rn(e, n, k, dtype=dtype, gen=gen, scale=k**-0.5)
    up = _rn(e, n, k, dtype=dtype, gen=gen, scale=k**-0.5)
    fused = moe_mod._fused_gate_up(x, gate, up)
    assert fused is not None and fused.shape == (e, t, n)
    separate = moe_mod._silu_mul(moe_mod._expert_bmm(x, gate, 0), moe_mod._expert_bmm(x, up, 0))
    assert torch.equal(fused, separate)
    # segmented: rows split unevenly over the experts (one segment empty)
    cuts = sorted({0, t} | {int(v) for v in torch.randint(0, t + 1, (e - 1,), generator=torch.Generator().manual_seed(t)).tolist()})
    while len(cuts) < e + 1:
        cuts.insert(1, 0)
    seg = torch.tensor(cuts, dtype=torch.int32, device="cuda")
    fused_seg = moe_mod._fused_gate_up(x, gate, up, seg)
    sep_seg = moe_mod._silu_mul(moe_mod._segmented_mm(x, gate, seg), moe_mod._segmented_mm(x, up, seg))
    for s in range(e):
        lo, hi = cuts[s], cuts[s + 1]
        assert torch.equal(fused_seg[lo:hi], sep_seg[lo:hi]), s
        assert torch.equal(fused_seg[lo:hi], separate[s, lo:hi]), s


@pytest.mark.parametrize("dtype", HALF)
def test_moe_equals_unfused_reference_schedule(dtype):
    """Fused sparse MoE == the reference's schedule run op by op (dense
    gate and up GEMMs, silu*up, dense down GEMM, route sum)."""
    gen = torch.Generator(device="cuda").manual_seed(4242)
    t, e, k, d, i = 333, 6, 2, 256, 320
    h = _rn(t, d, dtype=dtype, gen=gen)
    gate = _rn(e, i, d, dtype=dtype, gen=gen, scale=d**-0.5)
    up = _rn(e, i, d, dtype=dtype, gen=gen, scale=d**-0.5)
    down = _rn(e, d, i, dtype=dtype, gen=gen, scale=i**-0.5)
    sel = torch.topk(torch.randn(t, e, device="cuda", generator=gen), k).indices
    w = torch.rand(t, k, device="cuda", generator=gen).to(dtype)
    act = moe_mod._silu_mul(moe_mod._expert_bmm(h, gate, 0), moe_mod._expert_bmm(h, up, 0))
    y = moe_mod._expert_bmm(act, down, act.stride(0))
    out = torch.empty(t, d, device="cuda", dtype=dtype)
    lib = _lib.load()
    _lib.check(lib.bio_moe_route_sum(_lib.DTYPE_CODE[dtype], ctypes.c_void_p(y.data_ptr()),
                                     _lib.DTYPE_CODE[dtype], ctypes.c_void_p(w.data_ptr()),
                                     ctypes.c_void_p(sel.contiguous().data_ptr()),
                                     ctypes.c_void_p(out.data_ptr()), e, t, k, d, 0,
                                     _lib.stream_of(h)), "bio_moe_route_sum")
    assert torch.equal(deterministic_token_choice_moe(h, w, sel, gate, up, down), out)
