"""GPU parity and batch-invariance tests of the GEMM family (mm, addmm, linear, bmm).

Mirrors test_batch_invariance.py:42-172 of the reference suite and adds the
BASELINE sweep geometry (K = 4096, N in {4096, 11008}, M from 1 to 2048)
checked bitwise row-by-row and against the fp64 oracle.
"""

from __future__ import annotations

from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from batch_invariant_ops import bmm_persistent, linear_batch_invariant, matmul_persistent
from conftest import DTYPES, TOLERANCES, assert_first_sample_equal
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _randn(*shape, dtype, gen, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=gen) * scale).to(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 3, 5, 17))
def test_mm_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(1000 + batch_size)
    inputs = _randn(batch_size, 257, dtype=dtype, gen=gen)
    weight = _randn(257, 129, dtype=dtype, gen=gen)
    assert_first_sample_equal(matmul_persistent(inputs[:1], weight), matmul_persistent(inputs, weight))


@pytest.mark.parametrize("dtype", DTYPES)
def test_mm_matches_oracle(dtype):
    gen = torch.Generator(device="cuda").manual_seed(2000)
    left = _randn(37, 257, dtype=dtype, gen=gen)
    right = _randn(257, 91, dtype=dtype, gen=gen)
    out = matmul_persistent(left, right)
    torch.testing.assert_close(out.double().cpu(), O.mm(left, right), **TOLERANCES[dtype])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 5, 17))
def test_rank3_linear_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(2500 + batch_size)
    inputs = _randn(batch_size, 37, 257, dtype=dtype, gen=gen)
    weight = _randn(91, 257, dtype=dtype, gen=gen)
    bias = _randn(91, dtype=dtype, gen=gen)
    assert_first_sample_equal(
        linear_batch_invariant(inputs[:1], weight, bias), linear_batch_invariant(inputs, weight, bias)
    )


@pytest.mark.parametrize("dtype", DTYPES)
def test_linear_matches_torch_and_oracle(dtype):
    gen = torch.Generator(device="cuda").manual_seed(2700)
    inputs = _randn(3, 37, 257, dtype=dtype, gen=gen)
    weight = _randn(91, 257, dtype=dtype, gen=gen)
    bias = _randn(91, dtype=dtype, gen=gen)
    out = linear_batch_invariant(inputs, weight, bias)
    tol = {"rtol": 2e-2, "atol": 1.5e-1} if dtype == torch.bfloat16 else TOLERANCES[dtype]
    torch.testing.assert_close(out, F.linear(inputs, weight, bias), **tol)
    torch.testing.assert_close(out.double().cpu(), O.linear(inputs, weight, bias), **tol)


def test_projector_shape_is_batch_invariant():
    gen = torch.Generator(device="cuda").manual_seed(2750)
    inputs = _randn(2, 256, 1024, dtype=torch.bfloat16, gen=gen)
    weight = _randn(4096, 1024, dtype=torch.bfloat16, gen=gen)
    bias = _randn(4096, dtype=torch.bfloat16, gen=gen)
    assert_first_sample_equal(
        linear_batch_invariant(inputs[:1], weight, bias), linear_batch_invariant(inputs, weight, bias)
    )


def test_fp32_fov_projection_is_batch_invariant():
    gen = torch.Generator(device="cuda").manual_seed(2775)
    inputs = _randn(2, 2304, dtype=torch.float32, gen=gen)
    weight = _randn(2304, 2304, dtype=torch.float32, gen=gen)
    bias = _randn(2304, dtype=torch.float32, gen=gen)
    assert_first_sample_equal(
        linear_batch_invariant(inputs[:1], weight, bias), linear_batch_invariant(inputs, weight, bias)
    )


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 3, 5, 17))
def test_bmm_is_batch_invariant(dtype, batch_size):
    gen = torch.Generator(device="cuda").manual_seed(3000 + batch_size)
    left = _randn(batch_size, 33, 65, dtype=dtype, gen=gen)
    right = _randn(batch_size, 65, 47, dtype=dtype, gen=gen)
    assert_first_sample_equal(bmm_persistent(left[:1], right[:1]), bmm_persistent(left, right))


@pytest.mark.parametrize("dtype", DTYPES)
def test_bmm_matches_oracle_for_noncontiguous_attention_inputs(dtype):
    gen = torch.Generator(device="cuda").manual_seed(4000)
    query = _randn(4, 8, 33, 65, dtype=dtype, gen=gen).reshape(-1, 33, 65)
    key = _randn(4, 8, 47, 65, dtype=dtype, gen=gen).reshape(-1, 47, 65).transpose(1, 2)
    out = bmm_persistent(query, key)
    torch.testing.assert_close(out, torch.bmm(query, key), **TOLERANCES[dtype])
    torch.testing.assert_close(out.double().cpu(), O.bmm(query, key), **TOLERANCES[dtype])


def test_bmm_supports_more_than_cuda_grid_y_limit():
    gen = torch.Generator(device="cuda").manual_seed(4500)
    left = _randn(70_000, 1, 4, dtype=torch.bfloat16, gen=gen)
    right = _randn(70_000, 4, 1, dtype=torch.bfloat16, gen=gen)
    batched = bmm_persistent(left, right)
    assert_first_sample_equal(bmm_persistent(left[:1], right[:1]), batched)
    torch.testing.assert_close(batched.double().cpu(), O.bmm(left, right), **TOLERANCES[torch.bfloat16])


def test_bmm_broadcast_weight_stride_zero():
    gen = torch.Generator(device="cuda").manual_seed(4600)
    x = _randn(6, 40, 64, dtype=torch.bfloat16, gen=gen)
    w = _randn(64, 96, dtype=torch.bfloat16, gen=gen).unsqueeze(0).expand(6, -1, -1)
    out = bmm_persistent(x, w)
    torch.testing.assert_close(out.double().cpu(), O.bmm(x, w), **TOLERANCES[torch.bfloat16])
    assert_first_sample_equal(bmm_persistent(x[:1], w[:1]), out)


@pytest.mark.parametrize(
    "name", ["mm_f32", "addmm_f32", "linear_f32", "bmm_f32", "mm_f16", "addmm_f16", "linear_f16", "bmm_f16"]
)
def test_gemm_matches_reference_golden(name):
    case = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    x = {k: v.cuda() for k, v in case["inputs"].items()}
    if case["op"] == "mm":
        out = matmul_persistent(x["a"], x["b"], x.get("bias"))
    elif case["op"] == "linear":
        out = linear_batch_invariant(x["x"], x["weight"], x["bias"])
    else:
        out = bmm_persistent(x["a"], x["b"])
    golden = case["output"]
    tol = dict(TOLERANCES[golden.dtype])
    if golden.dtype == torch.float16:
        tol = {"rtol": 2e-3, "atol": 2e-2}
    torch.testing.assert_close(out.cpu(), golden, **tol)


# ---- BASELINE config 2 geometry: bf16 linear sweep, bitwise per row ------
@pytest.mark.parametrize("n", (4096, 11008))
@pytest.mark.parametrize("layout", ("linear", "addmm"))
def test_sweep_rows_are_bitwise_invariant(n, layout):
    gen = torch.Generator(device="cuda").manual_seed(n)
    k = 4096
    x = torch.randn(2048, k, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=gen) / 64).to(torch.bfloat16)
    bias = (torch.randn(n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    if layout == "linear":
        run = lambda rows: linear_batch_invariant(rows, w, bias)  # noqa: E731
    else:
        wt = w.t().contiguous()  # [K, N] row-major: N-contiguous B operand
        run = lambda rows: matmul_persistent(rows, wt, bias)  # noqa: E731
    full = run(x)
    for m in (1, 8, 32, 127, 128, 129, 512):
        part = run(x[:m])
        assert torch.equal(part, full[:m]), f"M={m} rows differ from the M=2048 run"
    # an unrelated companion batch: the first row must not move
    other = torch.cat([x[:1], torch.randn(300, k, device="cuda", generator=gen).to(torch.bfloat16)])
    assert torch.equal(run(other)[:1], full[:1])
    rows = [0, 1, 127, 128, 2047]
    ref = O.linear(x[rows], w, bias)
    torch.testing.assert_close(full[rows].double().cpu(), ref, rtol=1e-2, atol=1e-2)


def test_fp32_linspace_config1_is_batch_invariant():
    """BASELINE config 1 (README.md:63-76 of the reference): fp32 linspace mm."""
    b, d = 2048, 4096
    a = torch.linspace(-100, 100, b * d, device="cuda").reshape(b, d)
    w = torch.linspace(-100, 100, d * d, device="cuda").reshape(d, d)
    full = matmul_persistent(a, w)
    assert torch.equal(matmul_persistent(a[:1], w), full[:1])
    rows = [0, 1, 1000, 2047]
    ref = O.mm(a[rows], w)
    err = (full[rows].double().cpu() - ref).norm() / ref.norm()
    assert err < 1e-5, err


def test_odd_shapes_and_empty():
    gen = torch.Generator(device="cuda").manual_seed(77)
    for m, k, n in ((1, 1, 1), (3, 5, 7), (130, 65, 257), (5, 0, 9)):
        a = _randn(m, k, dtype=torch.bfloat16, gen=gen)
        b = _randn(k, n, dtype=torch.bfloat16, gen=gen)
        out = matmul_persistent(a, b)
        torch.testing.assert_close(out.double().cpu(), O.mm(a, b), rtol=2e-2, atol=2e-2)
    empty = matmul_persistent(torch.empty(0, 8, device="cuda"), torch.randn(8, 3, device="cuda"))
    assert empty.shape == (0, 3)


# ------------------------------------------------------------------ tile independence
# Every output tile runs the same per-element arithmetic (64-wide K blocks in
# order, four K=16 tensor-core MMAs each, fp32 accumulator, one rounding), so
# the tile shape -- one CTA (128 rows) or a CTA pair (256 rows), 32..256
# columns -- must not change a single bit.  Inputs span 2^-8..2^8 in
# magnitude so that accumulation order differences would show.
_TILES_K_MAJOR = ((128, 32), (128, 64), (128, 96), (128, 128), (128, 256), (256, 128), (256, 256))
_TILES_N_MAJOR = ((128, 64), (128, 128), (128, 256), (256, 128), (256, 256))


def _wide(*shape, dtype, gen, span):
    x = torch.randn(*shape, device="cuda", generator=gen)
    e = torch.randint(-span, span + 1, shape, device="cuda", generator=gen).float()
    return (x * torch.exp2(e)).to(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", ((1, 200, 64), (37, 512, 1000), (300, 384, 4096), (129, 96, 72)))
@pytest.mark.parametrize("b_layout", ("k_major", "n_major"))
@pytest.mark.parametrize("with_bias", (False, True))
def test_every_tile_shape_gives_identical_bits(dtype, m, n, k, b_layout, with_bias):
    from batch_invariant_ops import _gemm

    gen = torch.Generator(device="cuda").manual_seed(m * 7919 + n * 31 + k)
    span = 8 if dtype == torch.bfloat16 else 3
    a = _wide(m, k, dtype=dtype, gen=gen, span=span)
    if b_layout == "k_major":
        b = _wide(n, k, dtype=dtype, gen=gen, span=span).t()
        tiles = _TILES_K_MAJOR
    else:
        b = _wide(k, n, dtype=dtype, gen=gen, span=span)
        tiles = _TILES_N_MAJOR
    bias = _wide(n, dtype=dtype, gen=gen, span=2) if with_bias else None
    ref = _gemm.mm(a, b, bias, tile=(256, 256))
    for tile in tiles:
        out = _gemm.mm(a, b, bias, tile=tile)
        assert torch.equal(out, ref), f"tile {tile} differs from (256, 256)"
    expect = O.linear(a, b.t(), bias)
    tol = dict(TOLERANCES[dtype])
    scale = float(expect.abs().max()) + 1.0
    torch.testing.assert_close(ref.double().cpu(), expect, rtol=tol["rtol"], atol=tol["atol"] * scale)


@pytest.mark.parametrize("n", (4096, 11008, 16384))
def test_policy_tiles_at_sweep_switch_points_give_identical_bits(n):
    """The tile bio_gemm runs depends on M (bio_gemm_tile_for).  For every M of
    the config-2 sweep and its switch points, collect the tile the policy
    picks; then run EVERY one of those tiles on the same 8192-row input and
    require identical bits, and require that the policy's own run at each M
    gives exactly the rows of the full run."""
    from batch_invariant_ops import _gemm

    gen = torch.Generator(device="cuda").manual_seed(61_000 + n)
    k = 4096
    x = _wide(8192, k, dtype=torch.bfloat16, gen=gen, span=6)
    w = (torch.randn(n, k, device="cuda", generator=gen) / 64).to(torch.bfloat16)
    bias = (torch.randn(n, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ms = (1, 8, 32, 127, 128, 129, 255, 256, 257, 512, 2048, 8192)
    picked = {m: _gemm.tile_for(m, n, 1, sms) for m in ms}
    full = linear_batch_invariant(x, w, bias)
    for tile in sorted(set(picked.values())):
        out = _gemm.mm(x, w.t(), bias, tile=tile)
        assert torch.equal(out, full), f"N={n}: tile {tile} differs from the library's run"
    for m in ms:
        part = linear_batch_invariant(x[:m], w, bias)
        assert torch.equal(part, full[:m]), f"N={n}: M={m} (tile {picked[m]}) differs"


def test_unsupported_tile_is_rejected():
    from batch_invariant_ops import _gemm

    a = torch.randn(4, 64, device="cuda").bfloat16()
    b = torch.randn(64, 128, device="cuda").bfloat16()
    with pytest.raises(RuntimeError):
        _gemm.mm(a, b, tile=(128, 48))
    with pytest.raises(RuntimeError):
        _gemm.mm(a, b, tile=(128, 32))  # N-contiguous B needs tile_n >= 64


# ------------------------------------------------------------------ exact-slice fp32
# fp32 GEMMs run on the int8 tensor cores with exact integer slices
# (bio_gemm_f32_exact).  Bar: normwise error against fp64 <= 1e-6 (the fp32
# parity bar is 1e-5), agreement with the fp64-accumulating kernel, and the
# usual bitwise batch invariance.
def _normwise(out, ref):
    return float((out.double().cpu() - ref).norm() / ref.norm())


@pytest.mark.parametrize("m,n,k", ((1, 77, 64), (37, 300, 1000), (256, 512, 4096), (130, 129, 131)))
@pytest.mark.parametrize("b_layout", ("k_major", "n_major"))
def test_exact_f32_matches_fp64(m, n, k, b_layout):
    from batch_invariant_ops import _gemm

    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=gen) * 3
    if b_layout == "k_major":
        b = torch.randn(n, k, device="cuda", generator=gen).t()
    else:
        b = torch.randn(k, n, device="cuda", generator=gen)
    bias = torch.randn(n, device="cuda", generator=gen)
    ref = a.double().cpu() @ b.double().cpu() + bias.double().cpu()
    exact = _gemm.mm(a, b, bias)
    dfma = _gemm.mm(a, b, bias, exact_f32=False)
    assert _normwise(exact, ref) <= 1e-6
    assert _normwise(dfma, ref) <= 1e-6
    # elementwise: the exact-slice bound K * 2^-26 * max|A| * max|B|
    bound = k * 2.0**-26 * float(a.abs().max()) * float(b.abs().max())
    err = (exact.double().cpu() - ref).abs().max().item()
    assert err <= bound, (err, bound)
    assert torch.equal(_gemm.mm(a[:1], b, bias), exact[:1])


def test_exact_f32_linspace_config1_accuracy():
    # BASELINE config 1 at full size: massive cancellation, 1e-5 bar
    bsz, d = 2048, 4096
    a = torch.linspace(-100, 100, bsz * d, device="cuda").reshape(bsz, d)
    w = torch.linspace(-100, 100, d * d, device="cuda").reshape(d, d)
    out = matmul_persistent(a, w)
    rows = torch.tensor([0, 1, 1023, 2047])
    ref = a[rows].double().cpu() @ w.double().cpu()
    # the fp32 bar is 1e-5; the slices give ~1.6e-6 on this cancelling case
    # (every fp32 accumulation order gives 2e-4-5e-4)
    assert _normwise(out[rows], ref) <= 5e-6
    assert torch.equal(matmul_persistent(a[:1], w), out[:1])
    assert torch.equal(matmul_persistent(a[2047:], w), out[2047:])


def test_exact_f32_nonfinite_rows_give_nan():
    from batch_invariant_ops import _gemm

    a = torch.randn(4, 256, device="cuda")
    b = torch.randn(256, 64, device="cuda")
    a[2, 5] = float("inf")
    out = _gemm.mm(a, b)
    assert torch.isnan(out[2]).all()
    ref = a.double().cpu() @ b.double().cpu()
    assert _normwise(out[[0, 1, 3]], ref[[0, 1, 3]]) <= 1e-6


def test_exact_f32_batched_and_broadcast():
    gen = torch.Generator(device="cuda").manual_seed(99)
    a = torch.randn(6, 33, 200, device="cuda", generator=gen)
    w = torch.randn(200, 70, device="cuda", generator=gen)
    wb = w.unsqueeze(0).expand(6, 200, 70)  # stride-0 batch
    out = bmm_persistent(a, wb)
    ref = torch.bmm(a.double().cpu(), wb.double().cpu())
    assert _normwise(out, ref) <= 1e-6
    assert torch.equal(bmm_persistent(a[2:3], wb[2:3]), out[2:3])


def test_fp32_long_k_uses_fp64_accumulation_kernel():
    # K > 65536 is outside the exact-slice path (int32 headroom); bio_gemm's
    # fp64-accumulating kernel takes it
    gen = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(3, 70000, device="cuda", generator=gen)
    b = torch.randn(70000, 17, device="cuda", generator=gen)
    out = matmul_persistent(a, b)
    ref = a.double().cpu() @ b.double().cpu()
    assert _normwise(out, ref) <= 1e-6
