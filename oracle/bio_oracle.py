"""fp64 CPU oracle for the batch-invariant operator path.

TEST INFRASTRUCTURE ONLY.  This module restates, in float64 on the CPU, the
algorithm of each operator of yiannisha/robotics-batch-invariant-ops
(``batch_invariant_ops/batch_invariant_ops.py`` and ``batch_invariant_ops/moe.py``;
citations are ``file:line`` into that project).  It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` as the checker; the product path never calls it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by running the reference itself (its Triton
kernels under ``TRITON_INTERPRET=1``, its CPU MoE branch) with
``tests/golden/make_golden.py``.

All functions take and return torch tensors; inputs of any dtype/device are
copied to CPU float64 first.  Outputs are float64 (callers compare against
the kernel output with a tolerance).
"""

from __future__ import annotations

import math
from typing import Sequence

import torch


def _f64(x: torch.Tensor | None) -> torch.Tensor | None:
    if x is None:
        return None
    return x.detach().to(device="cpu", dtype=torch.float64)


# ---------------------------------------------------------------------------
# GEMM family
# ---------------------------------------------------------------------------
def mm(a, b, bias=None):
    """C = A B (+ bias after the full K reduction).

    batch_invariant_ops.py:61-139 (kernel; bias added to the fp32 accumulator
    at :134-138) and :271-343 (launcher)."""
    out = _f64(a) @ _f64(b)
    if bias is not None:
        out = out + _f64(bias)
    return out


def linear(x, weight, bias=None):
    """batch_invariant_ops.py:1608-1616: flatten leading dims, mm with W^T."""
    x64 = _f64(x)
    out = mm(x64.reshape(-1, x64.shape[-1]), _f64(weight).T, bias)
    return out.reshape(*x64.shape[:-1], weight.shape[0])


def bmm(a, b):
    """batch_invariant_ops.py:143-229, 346-431: independent GEMM per batch element."""
    return torch.bmm(_f64(a), _f64(b))


# ---------------------------------------------------------------------------
# Convolution family (im2col -> grouped GEMM, as the reference lowers it)
# ---------------------------------------------------------------------------
def _tuple(values, n: int) -> tuple[int, ...]:
    values = tuple(values) if isinstance(values, (tuple, list)) else (values,)
    if len(values) == 1:
        return values * n
    assert len(values) == n
    return tuple(int(v) for v in values)


def conv(x, weight, bias, stride, padding, dilation, groups):
    """N-d convolution (N = 1, 2, 3) by explicit im2col + grouped matmul.

    Follows conv1d_batch_invariant (:497-595, grouped path :566-595),
    conv2d_batch_invariant (:598-682, F.unfold im2col :640-667) and
    conv3d_batch_invariant (:685-780, padded as_strided im2col :731-760):
    patches[b, g, L, Cg*kvol] @ W[g, Cg*kvol, Og], bias after the reduction.
    The depthwise 1-D Triton kernel (:435-494) computes the same sum."""
    x64, w64 = _f64(x), _f64(weight)
    nd = w64.ndim - 2
    stride, padding, dilation = (_tuple(v, nd) for v in (stride, padding, dilation))
    batch, cin = x64.shape[:2]
    cout = w64.shape[0]
    ksize = tuple(w64.shape[2:])
    pad_spec = []
    for p in reversed(padding):
        pad_spec += [p, p]
    xp = torch.nn.functional.pad(x64, pad_spec)
    out_shape = tuple(
        (x64.shape[2 + i] + 2 * padding[i] - dilation[i] * (ksize[i] - 1) - 1) // stride[i] + 1
        for i in range(nd)
    )
    strides = xp.stride()
    patches = xp.as_strided(
        size=(batch, cin, *out_shape, *ksize),
        stride=(
            strides[0],
            strides[1],
            *(strides[2 + i] * stride[i] for i in range(nd)),
            *(strides[2 + i] * dilation[i] for i in range(nd)),
        ),
    )
    cg = cin // groups
    og = cout // groups
    kvol = math.prod(ksize)
    lvol = math.prod(out_shape)
    # [B, C, L..., k...] -> [B, G, L, Cg*kvol]
    perm = (0, *range(2, 2 + nd), 1, *range(2 + nd, 2 + 2 * nd))
    p = patches.permute(perm).reshape(batch, lvol, groups, cg * kvol).permute(0, 2, 1, 3)
    wg = w64.reshape(groups, og, cg * kvol).transpose(1, 2)  # [G, Cg*kvol, Og]
    out = torch.einsum("bglk,gko->bglo", p, wg)
    if bias is not None:
        out = out + _f64(bias).reshape(1, groups, 1, og)
    return out.permute(0, 1, 3, 2).reshape(batch, cout, *out_shape)


def conv_transpose(x, weight, bias, stride, groups):
    """Non-overlapping transposed convolution (stride == kernel, padding 0,
    dilation 1): per input position a grouped GEMM x[B*G, HW, Cg] @
    W[Cg, Og*kvol], then the pixel-shuffle layout transform.
    conv_transpose2d_batch_invariant :783-861, conv_transpose3d :864-941."""
    x64, w64 = _f64(x), _f64(weight)
    nd = w64.ndim - 2
    ksize = tuple(w64.shape[2:])
    assert _tuple(stride, nd) == ksize
    batch, cin = x64.shape[:2]
    spatial = tuple(x64.shape[2:])
    cg = cin // groups
    og = w64.shape[1]
    kvol = math.prod(ksize)
    xin = x64.reshape(batch, groups, cg, math.prod(spatial)).permute(0, 1, 3, 2)
    wg = w64.reshape(groups, cg, og * kvol)
    out = torch.einsum("bglc,gck->bglk", xin, wg)
    out = out.reshape(batch, groups, *spatial, og, *ksize)
    if bias is not None:
        out = out + _f64(bias).reshape(1, groups, *([1] * nd), og, *([1] * nd))
    # interleave: [B, G, Og, s0, k0, s1, k1, ...]
    perm = [0, 1, 2 + nd]
    for i in range(nd):
        perm += [2 + i, 3 + nd + i]
    out = out.permute(perm)
    return out.reshape(batch, groups * og, *(spatial[i] * ksize[i] for i in range(nd)))


# ---------------------------------------------------------------------------
# Row softmax family
# ---------------------------------------------------------------------------
def softmax(x, dim=-1):
    """Row softmax with the reference's edge rules (:1075-1114): an all -inf
    row gives max = -inf, every exponent 0, denominator 0 and output 0."""
    x64 = _f64(x)
    mx = x64.amax(dim=dim, keepdim=True)
    shifted = torch.where(torch.isneginf(mx), torch.full_like(x64, -math.inf), x64 - mx)
    e = torch.exp(shifted)
    den = e.sum(dim=dim, keepdim=True)
    return torch.where(den == 0, torch.zeros_like(e), e / torch.where(den == 0, 1.0, den))


def log_softmax(x, dim=-1):
    """x - max - log(sum(exp(x - max))) (:975-1034)."""
    x64 = _f64(x)
    mx = x64.amax(dim=dim, keepdim=True)
    return x64 - mx - torch.log(torch.exp(x64 - mx).sum(dim=dim, keepdim=True))


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
def sdpa(q, k, v, attn_mask=None, is_causal=False, scale=None, enable_gqa=False,
         query_rows=None):
    """Eager attention of scaled_dot_product_attention_batch_invariant
    (:1148-1213): GQA by repeating KV heads, top-left causal mask, boolean
    masks drop keys, float masks add; fully masked rows produce 0.

    ``query_rows`` (optional 1-D index tensor) evaluates only those query
    positions: the result is [..., len(query_rows), Dv], row r holding query
    position query_rows[r] with its causal/mask row at that absolute position
    (each query row is independent, so this is exactly the same arithmetic
    as the full evaluation restricted to those rows)."""
    q64, k64, v64 = _f64(q), _f64(k), _f64(v)
    lq_full = q64.shape[-2]
    rows = None
    if query_rows is not None:
        rows = torch.as_tensor(query_rows, dtype=torch.long).reshape(-1).cpu()
        q64 = q64.index_select(-2, rows)
    if enable_gqa:
        rep = q64.shape[-3] // k64.shape[-3]
        k64 = k64.repeat_interleave(rep, dim=-3)
        v64 = v64.repeat_interleave(rep, dim=-3)
    lk = k64.shape[-2]
    s = scale if scale is not None else 1.0 / math.sqrt(q64.shape[-1])
    scores = (q64 @ k64.transpose(-1, -2)) * s
    qpos = rows if rows is not None else torch.arange(lq_full)
    if is_causal:
        keep = torch.arange(lk)[None, :] <= qpos[:, None]
        scores = scores.masked_fill(~keep, -math.inf)
    elif attn_mask is not None:
        m = attn_mask.detach().cpu()
        if rows is not None and m.shape[-2] != 1:
            m = m.index_select(-2, rows)
        if m.dtype == torch.bool:
            scores = scores.masked_fill(~m, -math.inf)
        else:
            scores = scores + m.to(torch.float64)
    return softmax(scores, dim=-1) @ v64


def varlen_sdpa(q, k, v, cu_q, cu_kv, is_causal=False, causal_type=None, scale=None,
                query_tokens=None):
    """Packed-sequence attention (:1216-1344): each (q segment, kv segment)
    pair attends independently; rows outside every segment and segments with
    an empty KV range stay zero; TopLeft / BottomRight causal alignment.

    ``query_tokens`` (optional iterable of packed query token indices)
    evaluates only those tokens; the other rows of the result stay zero."""
    q64, k64, v64 = _f64(q), _f64(k), _f64(v)
    cq = [int(t) for t in cu_q.detach().cpu().tolist()]
    ck = [int(t) for t in cu_kv.detach().cpu().tolist()]
    out = torch.zeros(1, q64.shape[1], q64.shape[2], v64.shape[3], dtype=torch.float64)
    name = getattr(causal_type, "name", causal_type)
    if name is not None:
        name = str(name).rsplit(".", 1)[-1]
    wanted = None
    if query_tokens is not None:
        wanted = sorted({int(t) for t in query_tokens})
    for i in range(len(cq) - 1):
        qs, qe, ks, ke = cq[i], cq[i + 1], ck[i], ck[i + 1]
        lq, lk = qe - qs, ke - ks
        if lq == 0 or lk == 0:
            continue
        local = None
        if wanted is not None:
            local = [t - qs for t in wanted if qs <= t < qe]
            if not local:
                continue
        qpos = torch.tensor(local) if local is not None else torch.arange(lq)
        qi = q64[:, qs:qe].transpose(1, 2)
        ki = k64[:, ks:ke].transpose(1, 2)
        vi = v64[:, ks:ke].transpose(1, 2)
        mask = None
        causal = is_causal
        if is_causal and lq != lk:
            kidx = torch.arange(lk)[None, :]
            shift = lk - lq if name == "BottomRight" else 0
            mask = kidx <= torch.arange(lq)[:, None] + shift
            causal = False
        o = sdpa(qi, ki, vi, mask, causal, scale, enable_gqa=qi.shape[1] != ki.shape[1],
                 query_rows=qpos)
        out[:, qs + qpos] = o.transpose(1, 2)
    return out


# ---------------------------------------------------------------------------
# Reductions
# ---------------------------------------------------------------------------
def mean(x, dims: Sequence[int], keepdim=False):
    """Mean over `dims` (:1348-1482 single dim; :1643-1651 multi-dim)."""
    return _f64(x).mean(dim=tuple(dims), keepdim=keepdim)


def vector_norm(x, dims: Sequence[int] | None, keepdim=False):
    """sqrt(sum(x^2)) over `dims` (:1486-1597)."""
    x64 = _f64(x)
    if dims is None:
        dims = tuple(range(x64.ndim))
    return torch.sqrt((x64 * x64).sum(dim=tuple(dims), keepdim=keepdim))


# ---------------------------------------------------------------------------
# Fused normalisation (additions next to the path: the reference leaves
# layer norms to stock torch and builds RMSNorm from mean_dim, :1395-1482)
# ---------------------------------------------------------------------------
def layer_norm(x, normalized_ndim: int, weight=None, bias=None, eps=1e-5):
    """(x - mean) / sqrt(var + eps) * weight + bias over the trailing
    ``normalized_ndim`` dims, biased variance (torch.nn.functional.layer_norm)."""
    x64 = _f64(x)
    dims = tuple(range(x64.ndim - normalized_ndim, x64.ndim))
    mean = x64.mean(dim=dims, keepdim=True)
    var = ((x64 - mean) ** 2).mean(dim=dims, keepdim=True)
    out = (x64 - mean) / torch.sqrt(var + eps)
    if weight is not None:
        out = out * _f64(weight)
    if bias is not None:
        out = out + _f64(bias)
    return out


def rms_norm(x, normalized_ndim: int, weight=None, eps=None):
    """x / sqrt(mean(x^2) + eps) * weight over the trailing dims
    (torch.nn.functional.rms_norm; eps defaults to the fp32 epsilon)."""
    x64 = _f64(x)
    if eps is None:
        eps = torch.finfo(torch.float32).eps
    dims = tuple(range(x64.ndim - normalized_ndim, x64.ndim))
    out = x64 / torch.sqrt((x64 * x64).mean(dim=dims, keepdim=True) + eps)
    if weight is not None:
        out = out * _f64(weight)
    return out


def gated_linear(x, weight, activation="gelu_tanh"):
    """act(x W_g^T) * (x W_u^T) with weight [2F, K] = [W_g; W_u] (a transformer
    MLP's gated input projection; act = GELU in its tanh form, or silu).  No
    counterpart in the reference, which leaves MLP activations to stock torch."""
    y = linear(x, weight)
    f = y.shape[-1] // 2
    g, u = y[..., :f], y[..., f:]
    if activation == "gelu_tanh":
        act = 0.5 * g * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (g + 0.044715 * g ** 3)))
    else:
        act = g / (1.0 + torch.exp(-g))
    return act * u


# ---------------------------------------------------------------------------
# Mixture of experts
# ---------------------------------------------------------------------------
def moe(hidden, routing_weights, selected_experts, gate_w, up_w, down_w):
    """Top-k SwiGLU MoE (moe.py:11-92): for each token, sum over its k routes
    (left to right) of w * down(silu(gate h) * (up h)) of the selected expert.

    Evaluated per (route, expert) on the tokens that chose that expert, with
    each expert's weights widened to fp64 only while it is in use, so full
    model sizes (8 x 5632 x 2048 experts) fit in host memory."""
    h, w = _f64(hidden), _f64(routing_weights)
    sel = selected_experts.detach().cpu().long()
    tokens, top_k = sel.shape
    out = torch.zeros(tokens, h.shape[1], dtype=torch.float64)
    experts = gate_w.shape[0]
    for e in range(experts):
        hit = sel == e
        if not bool(hit.any()):
            continue
        g, u, d = _f64(gate_w[e]), _f64(up_w[e]), _f64(down_w[e])
        for j in range(top_k):
            idx = torch.nonzero(hit[:, j]).reshape(-1)
            if idx.numel() == 0:
                continue
            he = h.index_select(0, idx)
            inter = torch.nn.functional.silu(he @ g.T) * (he @ u.T)
            contrib = (inter @ d.T) * w.index_select(0, idx)[:, j : j + 1]
            out.index_add_(0, idx, contrib)
    return out


def moe_route_plan(selected_experts, experts):
    """Expected plan of the sparse MoE path: slots t*top_k + j sorted by
    expert, stably.  Returns (seg [E+1], slot_row [S] with -1 for ids outside
    [0, E), row_token [seg[E]]) as int64 tensors.  The dense evaluation that
    the sparse path must reproduce is moe.py:67-92 (``moe`` above)."""
    sel = selected_experts.detach().cpu().long().reshape(-1)
    top_k = selected_experts.shape[1] if selected_experts.ndim == 2 else 1
    valid = (sel >= 0) & (sel < experts)
    counts = torch.bincount(sel[valid], minlength=experts)
    seg = torch.zeros(experts + 1, dtype=torch.int64)
    seg[1:] = torch.cumsum(counts, 0)
    slot_row = torch.full_like(sel, -1)
    row_token = torch.zeros(int(seg[-1]), dtype=torch.int64)
    nxt = seg[:-1].clone()
    for i in range(sel.numel()):  # sequential: stable by construction
        e = int(sel[i])
        if 0 <= e < experts:
            slot_row[i] = nxt[e]
            row_token[nxt[e]] = i // top_k
            nxt[e] += 1
    return seg, slot_row, row_token


def topk_routing(logits, k):
    """Top-k expert choice with lowest-index tie-break and a softmax over the
    selected logits (the caller-side router of the MoE configs)."""
    l64 = _f64(logits)
    order = torch.argsort(-l64, dim=-1, stable=True)[:, :k]
    vals = torch.gather(l64, 1, order)
    return torch.softmax(vals, dim=-1), order
