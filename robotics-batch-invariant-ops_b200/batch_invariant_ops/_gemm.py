"""Host side of the batch-invariant GEMM: operand canonicalisation and launch.

Everything here goes straight to ``bio_gemm`` / ``bio_pack_rows`` in the
kernel library; no torch matmul is ever called (calling one from inside an
``aten::mm`` override would re-enter the override).

Operand rules of the tensor-core path (bf16/fp16): A is K-contiguous, B is K-
or N-contiguous, base pointers and row/batch strides are 16-byte aligned.
Operands that break a rule are first copied by ``bio_pack_rows`` into a dense
K-contiguous buffer whose K is padded with zeros to a multiple of 8.  The copy
is exact and the zero tail lies inside the last 64-wide K block that the
kernel zero-fills anyway, so packing never changes a result bit.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, tracing


def _ceil8(x: int) -> int:
    return (x + 7) // 8 * 8


@dataclass
class Operand:
    """A [batch1][batch2/div2][rows][cols] operand description (element strides)."""

    tensor: torch.Tensor  # keeps the storage alive for the launch
    ptr: int
    s_row: int
    s_col: int
    s1: int
    s2: int
    div2: int = 1


# Placeholder operand for K == 0 (the library fills C with the bias and never
# reads A or B).
_EMPTY = Operand(None, 0, 1, 1, 0, 0, 1)


def _aligned16(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def _pack(
    x: torch.Tensor,
    nb1: int,
    nb2: int,
    rows: int,
    cols: int,
    s_b1: int,
    s_b2: int,
    s_row: int,
    s_col: int,
) -> tuple[torch.Tensor, int]:
    """Dense [nb1, nb2, rows, cols_pad] copy of a strided operand."""
    cols_pad = _ceil8(max(cols, 1))
    out = torch.empty((nb1, nb2, rows, cols_pad), dtype=x.dtype, device=x.device)
    lib = _lib.load()
    _lib.check(
        lib.bio_pack_rows(
            _lib.DTYPE_CODE[x.dtype],
            ctypes.c_void_p(x.data_ptr()),
            nb1,
            nb2,
            rows,
            cols,
            s_b1,
            s_b2,
            s_row,
            s_col,
            ctypes.c_void_p(out.data_ptr()),
            cols_pad,
            x.device.index,
            _lib.stream_of(x),
        ),
        "bio_pack_rows",
    )
    return out, cols_pad


def operand_a(
    x: torch.Tensor,
    batch1: int,
    batch2: int,
    rows: int,
    k: int,
    s_row: int,
    s_k: int,
    s1: int,
    s2: int,
    div2: int = 1,
) -> Operand:
    """A operand (rows = M, cols = K) for the GEMM of ``x.dtype``."""
    if batch1 <= 1:
        s1 = 0 if batch1 == 1 else s1
    if rows == 1:
        s_row = _ceil8(k)
    if k == 1:
        s_k = 1
    if x.dtype == torch.float32:
        return Operand(x, x.data_ptr(), s_row, s_k, s1, s2, div2)
    common = s1 % 8 == 0 and s2 % 8 == 0 and _aligned16(x)
    if common and s_k == 1 and s_row % 8 == 0:
        return Operand(x, x.data_ptr(), s_row, 1, s1, s2, div2)
    if common and s_row == 1 and s_k % 8 == 0 and rows > 1:
        return Operand(x, x.data_ptr(), 1, s_k, s1, s2, div2)
    nb1 = 1 if s1 == 0 else batch1
    nb2 = 1 if s2 == 0 else (batch2 + div2 - 1) // div2
    packed, kp = _pack(x, nb1, nb2, rows, k, s1, s2, s_row, s_k)
    return Operand(
        packed,
        packed.data_ptr(),
        kp,
        1,
        0 if s1 == 0 else nb2 * rows * kp,
        0 if s2 == 0 else rows * kp,
        div2,
    )


def operand_b(
    x: torch.Tensor,
    batch1: int,
    batch2: int,
    k: int,
    n: int,
    s_k: int,
    s_n: int,
    s1: int,
    s2: int,
    div2: int = 1,
) -> Operand:
    """B operand: element (k, n) at s_k*k + s_n*n.  ``s_row``/``s_col`` of the
    returned Operand are (s_k, s_n)."""
    if batch1 <= 1:
        s1 = 0 if batch1 == 1 else s1
    if n == 1 and k == 1:
        s_k, s_n = 1, 8
    elif n == 1:
        if s_k == 1:
            s_n = _ceil8(k)
    elif k == 1:
        if s_n == 1:
            s_k = _ceil8(n)
    if x.dtype == torch.float32:
        return Operand(x, x.data_ptr(), s_k, s_n, s1, s2, div2)
    common = s1 % 8 == 0 and s2 % 8 == 0 and _aligned16(x)
    if common and s_k == 1 and s_n % 8 == 0:
        return Operand(x, x.data_ptr(), 1, s_n, s1, s2, div2)
    if common and s_n == 1 and s_k % 8 == 0:
        return Operand(x, x.data_ptr(), s_k, 1, s1, s2, div2)
    nb1 = 1 if s1 == 0 else batch1
    nb2 = 1 if s2 == 0 else (batch2 + div2 - 1) // div2
    # pack as K-major: rows = n, cols = k
    packed, kp = _pack(x, nb1, nb2, n, k, s1, s2, s_n, s_k)
    return Operand(
        packed,
        packed.data_ptr(),
        1,
        kp,
        0 if s1 == 0 else nb2 * n * kp,
        0 if s2 == 0 else n * kp,
        div2,
    )


def launch(a: Operand, b: Operand, c: torch.Tensor, **kw) -> None:
    """Enqueue one GEMM (see _launch); inside tracing.record_launches the call
    is recorded with its algorithmic flops and bytes (and an NVTX range)."""
    pushed = False
    if tracing.active():
        m, n, k = kw["m"], kw["n"], kw["k"]
        b1, b2 = kw["batch1"], kw["batch2"]
        es = c.element_size()
        na = (b1 if a.s1 else 1) * (-(-b2 // max(a.div2, 1)) if a.s2 else 1)
        nb = (b1 if b.s1 else 1) * (-(-b2 // max(b.div2, 1)) if b.s2 else 1)
        mode = "swiglu" if kw.get("swiglu_up") is not None else (
            "segmented" if kw.get("segments") is not None else "gemm")
        pushed = tracing.note(
            "gemm", f"bio_{mode} [M={m}, N={n}, K={k}, batch={b1 * b2}]",
            2.0 * m * n * k * b1 * b2 * (2 if mode == "swiglu" else 1),
            es * (na * m * k + nb * k * n * (2 if mode == "swiglu" else 1) + b1 * b2 * m * n), es)
    try:
        _launch(a, b, c, **kw)
    finally:
        tracing.done(pushed)


def _launch(
    a: Operand,
    b: Operand,
    c: torch.Tensor,
    *,
    batch1: int,
    batch2: int,
    m: int,
    n: int,
    k: int,
    c_sm: int,
    c_sn: int,
    c_s1: int,
    c_s2: int,
    bias: torch.Tensor | None = None,
    bias_per_row: bool = False,
    bias_s2: int = 0,
    alpha: float = 1.0,
    tile: tuple[int, int] | None = None,
    exact_f32: bool = True,
    segments: torch.Tensor | None = None,
    swiglu_up: Operand | None = None,
    gate_gelu: bool = False,
    residual: torch.Tensor | None = None,
) -> None:
    """Enqueue one GEMM on the current stream of ``c``'s device.

    ``segments`` (device int32 [batch1 + 1] row offsets) selects
    bio_gemm_segmented: segment s owns rows [segments[s], segments[s+1]) of A
    and C and multiplies them by B batch s.  ``swiglu_up`` (an operand with
    the same layout as ``b``) selects bio_gemm_swiglu: C = silu(A·B) * (A·up)
    with the roundings of separate GEMMs and bio_silu_mul; with ``gate_gelu``
    the gate activation is GELU-tanh instead of silu (GeGLU).  ``residual``
    (a row-contiguous [M, N] tensor of C's dtype) selects bio_gemm_residual:
    C = residual + (A·B + bias) with the roundings of a linear and an add.

    fp32 runs on the int8 tensor cores with exact integer slices
    (bio_gemm_f32_exact, workspace from the caching allocator) whenever that
    path applies (K <= 32768), else on the fp64-accumulating kernel of
    bio_gemm; ``exact_f32=False`` forces the latter.  ``tile`` = (tile_m,
    tile_n) selects bio_gemm_tiled, an explicit output tile."""
    args = _lib.GemmArgs()
    args.dtype = _lib.DTYPE_CODE[c.dtype]
    args.flags = (_lib.BIO_GEMM_BIAS_PER_ROW if bias_per_row else 0) | (
        _lib.BIO_GEMM_GATE_GELU_TANH if gate_gelu else 0)
    args.batch1 = batch1
    args.batch2 = batch2
    args.m, args.n, args.k = m, n, k
    args.a = a.ptr
    args.a_sm, args.a_sk, args.a_s1, args.a_s2, args.a_div2 = (
        a.s_row,
        a.s_col,
        a.s1,
        a.s2,
        a.div2,
    )
    args.b = b.ptr
    args.b_sk, args.b_sn, args.b_s1, args.b_s2, args.b_div2 = (
        b.s_row,
        b.s_col,
        b.s1,
        b.s2,
        b.div2,
    )
    args.c = c.data_ptr()
    args.c_sm, args.c_sn, args.c_s1, args.c_s2 = c_sm, c_sn, c_s1, c_s2
    args.bias = bias.data_ptr() if bias is not None else None
    args.bias_s2 = bias_s2
    args.alpha = alpha
    args.device = c.device.index
    lib = _lib.load()
    if swiglu_up is not None:
        if (swiglu_up.s_row, swiglu_up.s_col, swiglu_up.s1, swiglu_up.s2) != (
            b.s_row, b.s_col, b.s1, b.s2
        ):
            raise ValueError("swiglu up operand must share the gate operand's layout")
        _lib.check(
            lib.bio_gemm_swiglu(
                ctypes.byref(args), ctypes.c_void_p(swiglu_up.ptr),
                ctypes.c_void_p(segments.data_ptr() if segments is not None else None),
                _lib.stream_of(c),
            ),
            "bio_gemm_swiglu",
        )
        return
    if segments is not None:
        _lib.check(
            lib.bio_gemm_segmented(
                ctypes.byref(args), ctypes.c_void_p(segments.data_ptr()), _lib.stream_of(c)
            ),
            "bio_gemm_segmented",
        )
        return
    if tile is None and c.dtype == torch.float32 and exact_f32:
        ws_bytes = lib.bio_gemm_f32_exact_workspace(ctypes.byref(args))
        if ws_bytes > 0:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=c.device)
            _lib.check(
                lib.bio_gemm_f32_exact(
                    ctypes.byref(args), ctypes.c_void_p(ws.data_ptr()), ws_bytes,
                    _lib.stream_of(c),
                ),
                "bio_gemm_f32_exact",
            )
            return
    if residual is not None:
        _lib.check(
            lib.bio_gemm_residual(ctypes.byref(args), ctypes.c_void_p(residual.data_ptr()),
                                  residual.stride(0), _lib.stream_of(c)),
            "bio_gemm_residual",
        )
        return
    if tile is None:
        _lib.check(lib.bio_gemm(ctypes.byref(args), _lib.stream_of(c)), "bio_gemm")
    else:
        _lib.check(
            _lib.load().bio_gemm_tiled(ctypes.byref(args), tile[0], tile[1], _lib.stream_of(c)),
            "bio_gemm_tiled",
        )


def mm(
    a: torch.Tensor,
    b: torch.Tensor,
    bias: torch.Tensor | None = None,
    tile: tuple[int, int] | None = None,
    exact_f32: bool = True,
    alpha: float = 1.0,
) -> torch.Tensor:
    """C[M,N] = alpha * A[M,K] @ B[K,N] (+ bias[N]); any strides.  ``tile`` forces an
    output tile (tests of tile independence); ``exact_f32=False`` runs fp32 on
    the fp64-accumulating kernel instead of the exact-slice tensor-core path."""
    m, k = a.shape
    n = b.shape[1]
    c = torch.empty((m, n), device=a.device, dtype=a.dtype)
    if m == 0 or n == 0:
        return c
    if bias is not None:
        bias = bias.to(a.dtype).contiguous()
    if k == 0:
        opa = opb = _EMPTY
    else:
        opa = operand_a(a, 1, 1, m, k, a.stride(0), a.stride(1), 0, 0)
        opb = operand_b(b, 1, 1, k, n, b.stride(0), b.stride(1), 0, 0)
    launch(
        opa, opb, c, batch1=1, batch2=1, m=m, n=n, k=k, c_sm=n, c_sn=1, c_s1=0, c_s2=0, bias=bias,
        tile=tile, exact_f32=exact_f32, alpha=alpha,
    )
    return c


def gated(x: torch.Tensor, weight: torch.Tensor, gelu: bool) -> torch.Tensor | None:
    """act(x @ weight[:F]^T) * (x @ weight[F:]^T) for x [M, K], weight [2F, K]
    (f16/bf16) in one fused GEMM (bio_gemm_swiglu; act = GELU-tanh or silu),
    with the rounding steps of the separate linear, activation and product.
    None when the two weight halves do not share one layout."""
    m, k = x.shape
    f = weight.shape[0] // 2
    out = torch.empty((m, f), device=x.device, dtype=x.dtype)
    if m == 0 or f == 0:
        return out
    gate, up = weight[:f], weight[f:]
    opa = operand_a(x, 1, 1, m, k, x.stride(0), x.stride(1), 0, 0)
    opg = operand_b(gate, 1, 1, k, f, gate.stride(1), gate.stride(0), 0, 0)
    opu = operand_b(up, 1, 1, k, f, up.stride(1), up.stride(0), 0, 0)
    if (opg.s_row, opg.s_col) != (opu.s_row, opu.s_col):
        return None
    launch(opa, opg, out, batch1=1, batch2=1, m=m, n=f, k=k, c_sm=f, c_sn=1, c_s1=0, c_s2=0,
           swiglu_up=opu, gate_gelu=gelu)
    return out


def linear_residual(r: torch.Tensor, x: torch.Tensor, w: torch.Tensor,
                    bias: torch.Tensor | None) -> torch.Tensor | None:
    """r + (x @ w^T + bias) for r [M, N], x [M, K], w [N, K] (f16/bf16) in one
    GEMM (bio_gemm_residual); None when the residual's rows are not
    contiguous."""
    m, k = x.shape
    n = w.shape[0]
    if r.stride(-1) != 1 or (m > 1 and r.stride(0) < n):
        return None
    out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    if m == 0 or n == 0:
        return out
    if bias is not None:
        bias = bias.to(x.dtype).contiguous()
    b = w.t()
    opa = operand_a(x, 1, 1, m, k, x.stride(0), x.stride(1), 0, 0)
    opb = operand_b(b, 1, 1, k, n, b.stride(0), b.stride(1), 0, 0)
    launch(opa, opb, out, batch1=1, batch2=1, m=m, n=n, k=k, c_sm=n, c_sn=1, c_s1=0, c_s2=0,
           bias=bias, residual=r)
    return out


def bmm(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0) -> torch.Tensor:
    """C[b] = A[b] @ B[b]; each batch element is an independent fixed-schedule GEMM."""
    nb, m, k = a.shape
    n = b.shape[2]
    c = torch.empty((nb, m, n), device=a.device, dtype=a.dtype)
    if nb == 0 or m == 0 or n == 0:
        return c
    if k == 0:
        opa = opb = _EMPTY
    else:
        opa = operand_a(a, nb, 1, m, k, a.stride(1), a.stride(2), a.stride(0), 0)
        opb = operand_b(b, nb, 1, k, n, b.stride(1), b.stride(2), b.stride(0), 0)
    launch(
        opa,
        opb,
        c,
        batch1=nb,
        batch2=1,
        m=m,
        n=n,
        k=k,
        c_sm=n,
        c_sn=1,
        c_s1=m * n,
        c_s2=0,
        alpha=alpha,
    )
    return c


def tile_for(m: int, n: int, batch: int = 1, sms: int = 148,
             b_n_contiguous: bool = False) -> tuple[int, int]:
    """(tile_m, tile_n) that bio_gemm runs for an m x n bf16/fp16 GEMM over
    ``batch`` products on a device with ``sms`` SMs."""
    tm, tn = ctypes.c_int32(0), ctypes.c_int32(0)
    _lib.check(_lib.load().bio_gemm_tile_for(m, n, batch, sms, int(b_n_contiguous),
                                             ctypes.byref(tm), ctypes.byref(tn)),
               "bio_gemm_tile_for")
    return tm.value, tn.value


def tile_config(n: int, k: int, dtype: torch.dtype) -> tuple[int, int, int]:
    """(block_m, block_n, block_k) the library uses for (n, k, dtype)."""
    code = _lib.load().bio_gemm_tile_config(n, k, _lib.DTYPE_CODE[dtype])
    return code // 1000000, (code // 1000) % 1000, code % 1000
