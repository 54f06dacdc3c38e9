"""Host side of the fused attention kernels (dense SDPA and varlen).

Both end in one C entry (``bio_attention`` / ``bio_attention_varlen``).
bf16/fp16 run the tcgen05 kernels: 128-row query tiles (two per CTA for long
queries) with S and O in TMEM, keys in fixed 128-key blocks, one softmax
thread per query row; fp32 runs a CUDA-core kernel with one warp per query
row.  Q/K/V are read through their strides, KV heads are shared for
grouped-query attention by index arithmetic and masks are applied through
broadcast strides, so no repeat_interleave, mask materialisation, score
tensor or host synchronisation is needed.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib, tracing


class _AttnArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_sb", ctypes.c_int64),
        ("q_sh", ctypes.c_int64),
        ("q_st", ctypes.c_int64),
        ("k_sb", ctypes.c_int64),
        ("k_sh", ctypes.c_int64),
        ("k_st", ctypes.c_int64),
        ("v_sb", ctypes.c_int64),
        ("v_sh", ctypes.c_int64),
        ("v_st", ctypes.c_int64),
        ("o_sb", ctypes.c_int64),
        ("o_sh", ctypes.c_int64),
        ("o_st", ctypes.c_int64),
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("lq", ctypes.c_int64),
        ("lk", ctypes.c_int64),
        ("d", ctypes.c_int32),
        ("dv", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("mask_kind", ctypes.c_int32),
        ("mask_dtype", ctypes.c_int32),
        ("mask", ctypes.c_void_p),
        ("m_sb", ctypes.c_int64),
        ("m_sh", ctypes.c_int64),
        ("m_sq", ctypes.c_int64),
        ("m_sk", ctypes.c_int64),
        ("cu_q", ctypes.c_void_p),
        ("cu_k", ctypes.c_void_p),
        ("cu_is64", ctypes.c_int32),
        ("nseq", ctypes.c_int64),
        ("workspace", ctypes.c_void_p),
    ]


MASK_NONE, MASK_BOOL, MASK_ADD = 0, 1, 2
CAUSAL = {"none": 0, "top_left": 1, "bottom_right": 2, "equal": 3}
MAX_HEAD_DIM = 256


def _dim_contiguous(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """[B, H, L, D] view whose non-unit strides are 16-byte multiples, with D
    contiguous and a 16-byte aligned base (what the tensor-core kernel reads
    with TMA).  Otherwise an exact copy with D padded to a multiple of 8; the
    kernel still reads only the first D columns."""
    ok = t.stride(-1) == 1 and t.data_ptr() % 16 == 0
    for size, stride in zip(t.shape[:-1], t.stride()[:-1]):
        if size > 1 and stride % 8 != 0:
            ok = False
    if ok:
        return t
    from . import _gemm

    b, h, l, d = t.shape
    packed, _ = _gemm._pack(t, b, h, l, d, t.stride(0), t.stride(1), t.stride(2), t.stride(3))
    return packed


def _check_head_dims(d: int, dv: int) -> None:
    if d > MAX_HEAD_DIM or dv > MAX_HEAD_DIM:
        raise ValueError(f"head dimensions above {MAX_HEAD_DIM} are not supported (got {d}, {dv})")


def sdpa(q, k, v, attn_mask, is_causal, scale):
    """q [..., H, Lq, D], k [..., Hkv, Lk, D], v [..., Hkv, Lk, Dv] -> [..., H, Lq, Dv]."""
    lead = q.shape[:-3]
    h, lq, d = q.shape[-3:]
    hkv, lk = k.shape[-3], k.shape[-2]
    dv = v.shape[-1]
    _check_head_dims(d, dv)
    if h % hkv:
        raise ValueError("invalid grouped-query attention head counts")
    nb = math.prod(lead)
    q4 = _dim_contiguous(q.reshape(nb, h, lq, d))
    k4 = _dim_contiguous(k.reshape(nb, hkv, lk, d))
    v4 = _dim_contiguous(v.reshape(nb, hkv, lk, dv))
    if q.dtype != torch.float32:
        q4, k4, v4 = _tma_ready(q4), _tma_ready(k4), _tma_ready(v4)
    # Stored token-major ([nb, Lq, H, Dv] memory, returned as the [nb, H, Lq, Dv]
    # view), as flash attention lays out its output, so that the usual
    # out.transpose(-3, -2).reshape(..., H * Dv) that follows is a view.
    out = torch.empty((nb, lq, h, dv), device=q.device, dtype=q.dtype).transpose(1, 2)
    if out.numel() == 0:
        return out.reshape(*lead, h, lq, dv)
    a = _AttnArgs()
    a.dtype = _lib.DTYPE_CODE[q.dtype]
    a.device = q.device.index
    a.q, a.k, a.v, a.o = q4.data_ptr(), k4.data_ptr(), v4.data_ptr(), out.data_ptr()
    a.q_sb, a.q_sh, a.q_st = q4.stride(0), q4.stride(1), q4.stride(2)
    a.k_sb, a.k_sh, a.k_st = k4.stride(0), k4.stride(1), k4.stride(2)
    a.v_sb, a.v_sh, a.v_st = v4.stride(0), v4.stride(1), v4.stride(2)
    a.o_sb, a.o_sh, a.o_st = out.stride(0), out.stride(1), out.stride(2)
    a.batch, a.heads, a.kv_heads = nb, h, hkv
    a.lq, a.lk, a.d, a.dv = lq, lk, d, dv
    a.scale = scale if scale is not None else 1.0 / math.sqrt(d)
    a.causal = CAUSAL["top_left"] if is_causal else CAUSAL["none"]
    a.mask_kind = MASK_NONE
    mask_keep = None
    if attn_mask is not None and not is_causal:
        m = attn_mask
        if m.dtype == torch.bool:
            m = m.view(torch.uint8)
            a.mask_kind = MASK_BOOL
        else:
            if m.dtype not in _lib.DTYPE_CODE:
                m = m.to(q.dtype)
            a.mask_kind = MASK_ADD
            a.mask_dtype = _lib.DTYPE_CODE[m.dtype]
        me = m.expand(*lead, h, lq, lk)
        try:
            me = me.view(nb, h, lq, lk)
        except RuntimeError:
            me = me.reshape(nb, h, lq, lk)
        mask_keep = me
        a.mask = me.data_ptr()
        a.m_sb, a.m_sh, a.m_sq, a.m_sk = me.stride()
    pushed = tracing.note(
        "attention", f"bio_attention [B={nb}, H={h}/{hkv}, Lq={lq}, Lk={lk}, D={d}/{dv}, "
        f"causal={int(bool(is_causal))}]",
        2.0 * nb * h * lq * lk * (d + dv) / (2 if is_causal else 1),
        q.element_size() * (q4.numel() + k4.numel() + v4.numel() + out.numel()),
        q.element_size()) if tracing.active() else False
    try:
        _lib.check(_lib.load().bio_attention(ctypes.byref(a), _lib.stream_of(q)), "bio_attention")
    finally:
        tracing.done(pushed)
    del mask_keep
    return out.reshape(*lead, h, lq, dv)


def varlen(q, k, v, cu_q, cu_k, *, is_causal, causal_name, scale):
    """Packed q [1, Tq, H, D], k/v [1, Tk, Hkv, D|Dv] -> [1, Tq, H, Dv]."""
    _, tq, h, d = q.shape
    _, tk, hkv, _ = k.shape
    dv = v.shape[3]
    _check_head_dims(d, dv)
    q3 = _dim_contiguous(q[0])
    k3 = _dim_contiguous(k[0])
    v3 = _dim_contiguous(v[0])
    half = q.dtype != torch.float32
    if half:
        # [T, H, D] -> [1(batch), H, T, D] views for the TMA check, back to [T, H, D]
        q3 = _tma_ready(q3.permute(1, 0, 2).unsqueeze(0))[0].permute(1, 0, 2)
        k3 = _tma_ready(k3.permute(1, 0, 2).unsqueeze(0))[0].permute(1, 0, 2)
        v3 = _tma_ready(v3.permute(1, 0, 2).unsqueeze(0))[0].permute(1, 0, 2)
    alloc = torch.zeros if half else torch.empty
    out = alloc((1, tq, h, dv), device=q.device, dtype=v.dtype)
    if out.numel() == 0:
        return out
    cu_k = cu_k.to(cu_q.dtype) if cu_k.dtype != cu_q.dtype else cu_k
    cu_q = cu_q.contiguous()
    cu_k = cu_k.contiguous()
    a = _AttnArgs()
    a.dtype = _lib.DTYPE_CODE[q.dtype]
    a.device = q.device.index
    a.q, a.k, a.v, a.o = q3.data_ptr(), k3.data_ptr(), v3.data_ptr(), out.data_ptr()
    a.q_sb, a.q_sh, a.q_st = 0, q3.stride(1), q3.stride(0)
    a.k_sb, a.k_sh, a.k_st = 0, k3.stride(1), k3.stride(0)
    a.v_sb, a.v_sh, a.v_st = 0, v3.stride(1), v3.stride(0)
    a.o_sb, a.o_sh, a.o_st = 0, out.stride(2), out.stride(1)
    a.batch, a.heads, a.kv_heads = 1, h, hkv
    a.lq, a.lk, a.d, a.dv = tq, tk, d, dv
    a.scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if not is_causal:
        a.causal = CAUSAL["none"]
    elif causal_name == "BottomRight":
        a.causal = CAUSAL["bottom_right"]
    elif causal_name == "DontCare":
        a.causal = CAUSAL["equal"]
    else:
        a.causal = CAUSAL["top_left"]
    a.mask_kind = MASK_NONE
    a.cu_q, a.cu_k = cu_q.data_ptr(), cu_k.data_ptr()
    a.cu_is64 = 1 if cu_q.dtype == torch.int64 else 0
    a.nseq = cu_q.numel() - 1
    workspace = None
    if half:
        workspace = torch.empty(2 * a.nseq + 1, dtype=torch.int32, device=q.device)
        a.workspace = workspace.data_ptr()
    _lib.check(
        _lib.load().bio_attention_varlen(ctypes.byref(a), _lib.stream_of(q)), "bio_attention_varlen"
    )
    return out
