"""Generate golden vectors by running the REFERENCE implementation on the CPU.

Run in a container where yiannisha/robotics-batch-invariant-ops is checked
out (path given by --reference).  Triton kernels run
under ``TRITON_INTERPRET=1`` on CPU tensors (fp32 / fp16 GEMMs, softmax,
log-softmax, attention, conv lowering, mean, vector norm); the MoE runs the
reference's own CPU branch (moe.py:80-83).  bf16 ``tl.dot`` is not exact
under the interpreter, so GEMM-based cases use fp32/fp16 only.

Each case is stored as ``<name>.pt`` = {"op", "kwargs", "inputs", "output"}
with small seeded inputs.  The files are committed; this script documents how
they were made and regenerates them.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402

OUT = Path(__file__).resolve().parent


def _save(name, op, inputs, output, **kwargs):
    torch.save(
        {"op": op, "kwargs": kwargs, "inputs": inputs, "output": output.detach().clone()},
        OUT / f"{name}.pt",
    )
    print(f"{name}: {tuple(output.shape)} {output.dtype}")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="reference checkout")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import triton  # noqa: F401

    import batch_invariant_ops.batch_invariant_ops as ref
    from batch_invariant_ops.moe import deterministic_token_choice_moe

    ref._current_accelerator_type = lambda: "cpu"  # NUM_SMS = CPU threads under the interpreter
    g = torch.Generator().manual_seed(20260101)

    def rn(*shape, dtype=torch.float32):
        return torch.randn(*shape, generator=g).to(dtype)

    # ---- GEMM family
    for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16")):
        a, b, bias = rn(37, 257, dtype=dt), rn(257, 91, dtype=dt), rn(91, dtype=dt)
        _save(f"mm_{tag}", "mm", {"a": a, "b": b}, ref.matmul_persistent(a, b))
        _save(f"addmm_{tag}", "mm", {"a": a, "b": b, "bias": bias}, ref.matmul_persistent(a, b, bias))
        x, w, bb = rn(3, 37, 257, dtype=dt), rn(91, 257, dtype=dt), rn(91, dtype=dt)
        _save(f"linear_{tag}", "linear", {"x": x, "weight": w, "bias": bb},
              ref.linear_batch_invariant(x, w, bb))
        q = rn(4, 8, 33, 65, dtype=dt).reshape(-1, 33, 65)
        k = rn(4, 8, 47, 65, dtype=dt).reshape(-1, 47, 65).transpose(1, 2)
        _save(f"bmm_{tag}", "bmm", {"a": q, "b": k}, ref.bmm_persistent(q, k))

    # ---- convolution family (fp32)
    conv_cases = [
        ("conv1d_dense", (3, 4, 19), (7, 4, 3), (1,), (0,), (1,), 1),
        ("conv1d_grouped", (2, 8, 23), (12, 2, 4), (2,), (3,), (2,), 4),
        ("conv1d_depthwise", (2, 16, 31), (16, 1, 4), (1,), (3,), (1,), 16),
        ("conv2d_dense", (3, 4, 13, 11), (7, 4, 3, 3), (1, 1), (0, 0), (1, 1), 1),
        ("conv2d_grouped", (2, 4, 13, 11), (6, 2, 3, 2), (2, 1), (1, 0), (2, 1), 2),
        ("conv2d_patch14", (2, 3, 28, 28), (32, 3, 14, 14), (14, 14), (0, 0), (1, 1), 1),
        ("conv3d_patch", (3, 3, 2, 16, 16), (12, 3, 2, 16, 16), (2, 16, 16), (0, 0, 0), (1, 1, 1), 1),
        ("conv3d_grouped", (2, 4, 7, 9, 8), (6, 2, 3, 2, 2), (2, 1, 2), (1, 0, 1), (2, 1, 1), 2),
    ]
    for name, xs, ws, st, pd, dl, gr in conv_cases:
        x, w, bias = rn(*xs), rn(*ws), rn(ws[0])
        nd = len(xs) - 2
        out = ref.convolution_batch_invariant(x, w, bias, st, pd, dl, False, (0,) * nd, gr)
        _save(name, "conv", {"x": x, "weight": w, "bias": bias}, out,
              stride=st, padding=pd, dilation=dl, groups=gr)
    for name, xs, ws, st, gr in [
        ("convT2d_g1", (2, 4, 3, 3), (4, 6, 2, 2), (2, 2), 1),
        ("convT2d_g2", (2, 4, 3, 3), (4, 3, 2, 2), (2, 2), 2),
        ("convT3d_g2", (2, 4, 2, 3, 3), (4, 3, 2, 2, 2), (2, 2, 2), 2),
        ("convT3d_411", (3, 8, 2, 3, 3), (8, 6, 4, 1, 1), (4, 1, 1), 1),
    ]:
        x, w = rn(*xs), rn(*ws)
        bias = rn(ws[1] * gr)
        nd = len(xs) - 2
        out = ref.convolution_batch_invariant(x, w, bias, st, (0,) * nd, (1,) * nd, True, (0,) * nd, gr)
        _save(name, "conv_transpose", {"x": x, "weight": w, "bias": bias}, out, stride=st, groups=gr)

    # ---- softmax / log_softmax
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        x = rn(3, 7, 145, dtype=dt)
        for dim in (-1, 1):
            _save(f"softmax_{tag}_d{dim % 3}", "softmax", {"x": x}, ref.softmax(x, dim=dim), dim=dim)
            _save(f"log_softmax_{tag}_d{dim % 3}", "log_softmax", {"x": x},
                  ref.log_softmax(x, dim=dim), dim=dim)
    x = rn(4, 2100)
    x[1] = -math.inf
    _save("softmax_f32_wide_neginf_row", "softmax", {"x": x}, ref.softmax(x, dim=-1), dim=-1)

    # ---- attention (fp32)
    q, k, v = rn(2, 8, 33, 65), rn(2, 8, 47, 65), rn(2, 8, 47, 39)
    for causal in (False, True):
        _save(f"sdpa_causal{int(causal)}", "sdpa", {"q": q, "k": k, "v": v},
              ref.scaled_dot_product_attention_batch_invariant(q, k, v, is_causal=causal),
              is_causal=causal)
    q, k, v = rn(2, 4, 17, 32), rn(2, 4, 23, 32), rn(2, 4, 23, 24)
    bmask = torch.rand(2, 1, 17, 23, generator=g) > 0.2
    bmask[:, :, -1] = False
    fmask = torch.where(bmask, torch.tensor(0.0), torch.tensor(-math.inf))
    _save("sdpa_boolmask", "sdpa", {"q": q, "k": k, "v": v, "attn_mask": bmask},
          ref.scaled_dot_product_attention_batch_invariant(q, k, v, attn_mask=bmask))
    _save("sdpa_floatmask", "sdpa", {"q": q, "k": k, "v": v, "attn_mask": fmask},
          ref.scaled_dot_product_attention_batch_invariant(q, k, v, attn_mask=fmask))
    q, k, v = rn(2, 8, 17, 32), rn(2, 2, 23, 32), rn(2, 2, 23, 24)
    _save("sdpa_gqa", "sdpa", {"q": q, "k": k, "v": v},
          ref.scaled_dot_product_attention_batch_invariant(q, k, v, enable_gqa=True, scale=0.3),
          enable_gqa=True, scale=0.3)

    # ---- varlen attention (fp32)
    q_lens, kv_lens = (5, 3, 7), (7, 4, 5)
    q, k, v = rn(1, sum(q_lens), 4, 32), rn(1, sum(kv_lens), 2, 32), rn(1, sum(kv_lens), 2, 24)
    cq = torch.tensor([0, 5, 8, 15], dtype=torch.int32)
    ck = torch.tensor([0, 7, 11, 16], dtype=torch.int32)
    for ct in (None, "TopLeft", "BottomRight"):
        out = ref.varlen_scaled_dot_product_attention_batch_invariant(
            q, k, v, cq, ck, is_causal=ct is not None, causal_type=ct)
        _save(f"varlen_{ct or 'none'}", "varlen", {"q": q, "k": k, "v": v, "cu_q": cq, "cu_kv": ck},
              out, is_causal=ct is not None, causal_type=ct)
    q = rn(1, 11, 2, 16)
    k, v = rn(1, 11, 2, 16), rn(1, 11, 2, 16)
    c = torch.tensor([0, 5, 9], dtype=torch.int32)
    _save("varlen_uncovered", "varlen", {"q": q, "k": k, "v": v, "cu_q": c, "cu_kv": c},
          ref.varlen_scaled_dot_product_attention_batch_invariant(q, k, v, c, c))
    cq = torch.tensor([0, 3, 6], dtype=torch.int32)
    ck = torch.tensor([0, 0, 4], dtype=torch.int32)
    q, k, v = rn(1, 6, 2, 16), rn(1, 4, 2, 16), rn(1, 4, 2, 16)
    _save("varlen_empty_kv", "varlen", {"q": q, "k": k, "v": v, "cu_q": cq, "cu_kv": ck},
          ref.varlen_scaled_dot_product_attention_batch_invariant(q, k, v, cq, ck, is_causal=True,
                                                                 causal_type="BottomRight"),
          is_causal=True, causal_type="BottomRight")

    # ---- mean / vector norm: the reference wrappers assert is_cuda, so the
    # golden values come from its Triton kernels launched directly with the
    # wrappers' own (M, N, K) view logic (:1395-1482, :1525-1597).
    def ref_mean(x, dim):
        shape = list(x.shape)
        M = math.prod(shape[:dim])
        N = shape[dim]
        K = math.prod(shape[dim + 1:])
        x3 = x.reshape(M, N, K)
        out = torch.empty(M, K, dtype=x.dtype)
        ref.mean_kernel[(M * K,)](x3, out, x3.stride(0), x3.stride(1), x3.stride(2),
                                  out.stride(0), out.stride(1), M, N, K, 1024)
        return out.reshape(shape[:dim] + shape[dim + 1:])

    def ref_norm(x, dims):
        dims = tuple(d % x.ndim for d in dims)
        kept = tuple(d for d in range(x.ndim) if d not in dims)
        R = math.prod(x.shape[d] for d in dims)
        M = math.prod(x.shape[d] for d in kept)
        xi = x.permute(*kept, *dims).contiguous().reshape(M, R, 1)
        out = torch.empty(M, dtype=x.dtype)
        ref._vector_norm_kernel[(triton.cdiv(M, 8),)](xi, out, xi.stride(0), xi.stride(1),
                                                       xi.stride(2), M, R, 1,
                                                       BLOCK_SIZE=1024, OUTPUT_BLOCK_SIZE=8)
        return out.reshape(tuple(x.shape[d] for d in kept))

    import triton
    x = rn(6, 2048)
    _save("mean_last", "mean", {"x": x}, ref_mean(x, 1), dims=(1,))
    x = rn(3, 17, 5, 11)
    _save("mean_mid", "mean", {"x": x}, ref_mean(x, 1), dims=(1,))
    for dims in ((1,), (1, 3), (0, 1, 2, 3)):
        _save(f"norm_{''.join(map(str, dims))}", "norm", {"x": x}, ref_norm(x, dims), dims=dims)

    # ---- MoE: the reference's own CPU branch (moe.py:80-83)
    hidden = rn(7, 12)
    gate, up, down = rn(5, 16, 12), rn(5, 16, 12), rn(5, 12, 16)
    sel = torch.randint(0, 5, (7, 3), generator=g)
    w = torch.rand(7, 3, generator=g)
    _save("moe_f32", "moe", {"hidden": hidden, "routing_weights": w, "selected_experts": sel,
                             "gate": gate, "up": up, "down": down},
          deterministic_token_choice_moe(hidden, w, sel, gate, up, down))


if __name__ == "__main__":
    main()
