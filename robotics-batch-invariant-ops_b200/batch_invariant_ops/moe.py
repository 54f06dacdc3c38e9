"""Deterministic token-choice mixture of experts (reference batch_invariant_ops/moe.py:11-92).

Two evaluation paths with identical results, bit for bit:

* sparse (bf16/fp16, up to 1024 experts): ``bio_moe_plan`` sorts the routed
  slots by expert (a stable counting sort, no atomic positions),
  ``bio_moe_gather_rows`` copies each routed token's row, three segmented
  expert GEMMs (``bio_gemm_segmented``) run only on the rows routed to each
  expert, and ``bio_moe_route_sum_sorted`` adds each token's routes left to
  right.  Work is top_k / experts of the dense path.
* dense (fp32, or more than 1024 experts), as the reference: every expert
  on every token through fixed-schedule batched GEMMs (tokens broadcast with
  a stride-0 batch), then ``bio_moe_route_sum`` gathers the routes.

Both apply ``bio_silu_mul`` between the GEMMs.  A GEMM output row depends
only on its own input row and the expert's weights, so computing a row among
the routed rows (sparse) or among all tokens (dense) gives the same bits, and
a token's output never depends on the other tokens or on the routing of the
batch.  No atomics in any accumulation.
"""

from __future__ import annotations

import ctypes

import torch

from . import _gemm, _lib


def _expert_bmm(x: torch.Tensor, w: torch.Tensor, x_batch_stride: int) -> torch.Tensor:
    """y[e] = x[e] @ w[e]^T for w [E, N, K]; x [E, T, K] given by strides."""
    e, n, k = w.shape
    t = x.shape[-2]
    y = torch.empty((e, t, n), device=x.device, dtype=x.dtype)
    if y.numel() == 0:
        return y
    if k == 0:
        y.zero_()
        return y
    opa = _gemm.operand_a(x, e, 1, t, k, x.stride(-2), x.stride(-1), x_batch_stride, 0)
    opb = _gemm.operand_b(w, e, 1, k, n, w.stride(2), w.stride(1), w.stride(0), 0)
    _gemm.launch(opa, opb, y, batch1=e, batch2=1, m=t, n=n, k=k, c_sm=n, c_sn=1, c_s1=t * n,
                 c_s2=0)
    return y


def _silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    act = torch.empty_like(gate)
    if act.numel() == 0:
        return act
    _lib.check(
        _lib.load().bio_silu_mul(
            _lib.DTYPE_CODE[gate.dtype],
            ctypes.c_void_p(gate.data_ptr()),
            ctypes.c_void_p(up.data_ptr()),
            ctypes.c_void_p(act.data_ptr()),
            act.numel(),
            gate.device.index,
            _lib.stream_of(gate),
        ),
        "bio_silu_mul",
    )
    return act


def _route_weights(routing_weights: torch.Tensor) -> torch.Tensor:
    weights = routing_weights.contiguous()
    if weights.dtype not in _lib.DTYPE_CODE:
        weights = weights.to(torch.float32)
    return weights


def _swiglu_operands(x, gate_weight, up_weight, rows, x_batch, x_s1):
    """(A, gate B, up B) operands for bio_gemm_swiglu, or None when the two
    weights do not end up with one layout (the separate path then runs)."""
    e, n, k = gate_weight.shape
    opa = _gemm.operand_a(x, e, 1, rows, k, x.stride(-2), x.stride(-1), x_s1, 0)
    opg = _gemm.operand_b(gate_weight, e, 1, k, n, gate_weight.stride(2), gate_weight.stride(1),
                          gate_weight.stride(0), 0)
    opu = _gemm.operand_b(up_weight, e, 1, k, n, up_weight.stride(2), up_weight.stride(1),
                          up_weight.stride(0), 0)
    if (opg.s_row, opg.s_col, opg.s1, opg.s2) != (opu.s_row, opu.s_col, opu.s1, opu.s2):
        return None
    return opa, opg, opu


def _fused_gate_up(x, gate_weight, up_weight, segments=None):
    """act = silu(x @ gate^T) * (x @ up^T) per expert in one fused GEMM
    (bio_gemm_swiglu), bit-identical to the separate GEMMs + bio_silu_mul.
    Dense: x [T, K] broadcast to every expert, act [E, T, N].  Segmented:
    x [S, K] in expert order, act [S, N].  None when not applicable."""
    e, n, k = gate_weight.shape
    if x.dtype not in (torch.float16, torch.bfloat16) or k == 0 or n == 0:
        return None
    rows = x.shape[0]
    ops = _swiglu_operands(x, gate_weight, up_weight, rows, e, 0)
    if ops is None:
        return None
    opa, opg, opu = ops
    if segments is None:
        act = torch.empty((e, rows, n), device=x.device, dtype=x.dtype)
        c_s1 = rows * n
    else:
        act = torch.empty((rows, n), device=x.device, dtype=x.dtype)
        c_s1 = 0
    if act.numel() == 0:
        return act
    _gemm.launch(opa, opg, act, batch1=e, batch2=1, m=rows, n=n, k=k, c_sm=n, c_sn=1,
                 c_s1=c_s1, c_s2=0, segments=segments, swiglu_up=opu)
    return act


def _dense_moe(h, routing_weights, sel, gate_weight, up_weight, down_weight) -> torch.Tensor:
    """Every expert on every token (the reference's schedule)."""
    num_experts, _, hidden_size = gate_weight.shape
    token_count, top_k = sel.shape
    act = _fused_gate_up(h, gate_weight, up_weight)
    if act is None:
        act = _silu_mul(_expert_bmm(h, gate_weight, 0), _expert_bmm(h, up_weight, 0))
    expert_out = _expert_bmm(act, down_weight, act.stride(0))
    weights = _route_weights(routing_weights)
    out = torch.empty((token_count, hidden_size), device=h.device, dtype=h.dtype)
    _lib.check(
        _lib.load().bio_moe_route_sum(
            _lib.DTYPE_CODE[h.dtype],
            ctypes.c_void_p(expert_out.data_ptr()),
            _lib.DTYPE_CODE[weights.dtype],
            ctypes.c_void_p(weights.data_ptr()),
            ctypes.c_void_p(sel.data_ptr()),
            ctypes.c_void_p(out.data_ptr()),
            num_experts,
            token_count,
            top_k,
            hidden_size,
            h.device.index,
            _lib.stream_of(h),
        ),
        "bio_moe_route_sum",
    )
    return out


def _segmented_mm(x: torch.Tensor, w: torch.Tensor, seg: torch.Tensor) -> torch.Tensor:
    """y[r] = x[r] @ w[e]^T for the rows r of segment e; x [S, K], w [E, N, K]."""
    e, n, k = w.shape
    rows = x.shape[0]
    y = torch.empty((rows, n), device=x.device, dtype=x.dtype)
    opa = _gemm.operand_a(x, e, 1, rows, k, x.stride(0), x.stride(1), 0, 0)
    opb = _gemm.operand_b(w, e, 1, k, n, w.stride(2), w.stride(1), w.stride(0), 0)
    _gemm.launch(opa, opb, y, batch1=e, batch2=1, m=rows, n=n, k=k, c_sm=n, c_sn=1, c_s1=0,
                 c_s2=0, segments=seg)
    return y


def _sparse_moe(h, routing_weights, sel, gate_weight, up_weight, down_weight) -> torch.Tensor:
    """Each expert on its routed tokens only (same bits as _dense_moe)."""
    num_experts, _, hidden_size = gate_weight.shape
    token_count, top_k = sel.shape
    lib = _lib.load()
    dev = h.device.index
    stream = _lib.stream_of(h)
    code = _lib.DTYPE_CODE[h.dtype]
    ws_bytes = lib.bio_moe_plan_workspace(num_experts, token_count, top_k)
    if ws_bytes <= 0:
        raise ValueError("routing shape not supported by the sparse path")
    plan = torch.empty(ws_bytes // 4, dtype=torch.int32, device=h.device)
    _lib.check(
        lib.bio_moe_plan(ctypes.c_void_p(sel.data_ptr()), num_experts, token_count, top_k,
                         ctypes.c_void_p(plan.data_ptr()), ws_bytes, dev, stream),
        "bio_moe_plan",
    )
    slots = token_count * top_k
    xs = torch.empty((slots, hidden_size), device=h.device, dtype=h.dtype)
    _lib.check(
        lib.bio_moe_gather_rows(code, ctypes.c_void_p(h.data_ptr()), hidden_size,
                                ctypes.c_void_p(plan.data_ptr()), num_experts, token_count,
                                top_k, ctypes.c_void_p(xs.data_ptr()), dev, stream),
        "bio_moe_gather_rows",
    )
    seg = plan[: num_experts + 1]
    act = _fused_gate_up(xs, gate_weight, up_weight, seg)
    if act is None:
        act = _silu_mul(_segmented_mm(xs, gate_weight, seg), _segmented_mm(xs, up_weight, seg))
    ys = _segmented_mm(act, down_weight, seg)
    weights = _route_weights(routing_weights)
    out = torch.empty((token_count, hidden_size), device=h.device, dtype=h.dtype)
    _lib.check(
        lib.bio_moe_route_sum_sorted(
            code, ctypes.c_void_p(ys.data_ptr()), _lib.DTYPE_CODE[weights.dtype],
            ctypes.c_void_p(weights.data_ptr()), ctypes.c_void_p(plan.data_ptr()),
            ctypes.c_void_p(out.data_ptr()), num_experts, token_count, top_k, hidden_size,
            dev, stream,
        ),
        "bio_moe_route_sum_sorted",
    )
    return out


def sparse_path_applies(dtype: torch.dtype, num_experts: int, token_count: int, top_k: int,
                        intermediate_size: int, hidden_size: int) -> bool:
    """Whether deterministic_token_choice_moe evaluates only the routed rows."""
    return (
        dtype in (torch.float16, torch.bfloat16)
        and 1 <= num_experts <= 1024
        and intermediate_size > 0
        and hidden_size > 0
        and token_count * top_k < 2**31
    )


def deterministic_token_choice_moe(
    hidden_states: torch.Tensor,
    routing_weights: torch.Tensor,
    selected_experts: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    down_weight: torch.Tensor,
    workspace: dict[str, torch.Tensor] | None = None,
) -> torch.Tensor:
    """Evaluate a top-k SwiGLU MoE without atomic routing or accumulation.

    ``gate_weight`` and ``up_weight`` have shape ``(E, I, D)`` and
    ``down_weight`` has shape ``(E, D, I)``.  ``workspace`` is accepted for
    drop-in compatibility and ignored (reference moe.py:28-32, :41).
    Out-of-range expert ids set BIO_DEV_INDEX in the library status word and
    zero the affected rows (the reference raises a device-side assert).
    """
    del workspace
    if hidden_states.ndim != 2:
        raise ValueError(
            f"hidden_states must have shape (tokens, hidden), got {hidden_states.shape}"
        )
    if routing_weights.ndim != 2 or selected_experts.shape != routing_weights.shape:
        raise ValueError(
            "routing_weights and selected_experts must have the same (tokens, top_k) shape"
        )
    if routing_weights.shape[0] != hidden_states.shape[0]:
        raise ValueError("routing tensors and hidden_states have different token counts")
    if gate_weight.ndim != 3 or up_weight.shape != gate_weight.shape:
        raise ValueError(
            "gate_weight and up_weight must have the same (experts, intermediate, hidden) shape"
        )
    num_experts, intermediate_size, hidden_size = gate_weight.shape
    if hidden_states.shape[1] != hidden_size:
        raise ValueError("hidden_states and expert weights have incompatible hidden dimensions")
    if down_weight.shape != (num_experts, hidden_size, intermediate_size):
        raise ValueError("down_weight must have shape (experts, hidden, intermediate)")
    token_count, top_k = selected_experts.shape
    if token_count == 0:
        return hidden_states.new_empty((0, hidden_size))
    if top_k == 0:
        return hidden_states.new_zeros((token_count, hidden_size))
    if not hidden_states.is_cuda:
        raise AssertionError("batch-invariant operators require CUDA tensors")
    dtype = hidden_states.dtype
    if dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"unsupported dtype: {dtype}")
    if not (gate_weight.dtype == up_weight.dtype == down_weight.dtype == dtype):
        raise ValueError("expert weights and hidden_states must have the same dtype")

    h = hidden_states if hidden_states.is_contiguous() else hidden_states.contiguous()
    sel = selected_experts.to(torch.int64).contiguous()
    if sparse_path_applies(dtype, num_experts, token_count, top_k, intermediate_size,
                           hidden_size):
        return _sparse_moe(h, routing_weights, sel, gate_weight, up_weight, down_weight)
    return _dense_moe(h, routing_weights, sel, gate_weight, up_weight, down_weight)
