"""Deterministic token-choice mixture of experts (reference batch_invariant_ops/moe.py:11-92).

Dense all-expert SwiGLU through three fixed-schedule expert GEMMs (tokens are
broadcast to every expert with a stride-0 batch, no copy), ``bio_silu_mul``
between them, then ``bio_moe_route_sum`` gathers each token's top-k routes and
adds them left to right.  No atomics anywhere, so a token's output is
independent of the other tokens and of the routing of the batch.
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

    h = hidden_states
    gate = _expert_bmm(h, gate_weight, 0)
    up = _expert_bmm(h, up_weight, 0)
    act = torch.empty_like(gate)
    lib = _lib.load()
    stream = _lib.stream_of(h)
    dev = h.device.index
    _lib.check(
        lib.bio_silu_mul(
            _lib.DTYPE_CODE[dtype],
            ctypes.c_void_p(gate.data_ptr()),
            ctypes.c_void_p(up.data_ptr()),
            ctypes.c_void_p(act.data_ptr()),
            act.numel(),
            dev,
            stream,
        ),
        "bio_silu_mul",
    )
    expert_out = _expert_bmm(act, down_weight, act.stride(0))
    weights = routing_weights.contiguous()
    if weights.dtype not in _lib.DTYPE_CODE:
        weights = weights.to(torch.float32)
    sel = selected_experts.to(torch.int64).contiguous()
    out = torch.empty((token_count, hidden_size), device=h.device, dtype=dtype)
    _lib.check(
        lib.bio_moe_route_sum(
            _lib.DTYPE_CODE[dtype],
            ctypes.c_void_p(expert_out.data_ptr()),
            _lib.DTYPE_CODE[weights.dtype],
            ctypes.c_void_p(weights.data_ptr()),
            ctypes.c_void_p(sel.data_ptr()),
            ctypes.c_void_p(out.data_ptr()),
            num_experts,
            token_count,
            top_k,
            hidden_size,
            dev,
            stream,
        ),
        "bio_moe_route_sum",
    )
    return out
