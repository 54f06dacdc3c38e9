"""bf16 parity against the reference's own Triton kernels on the B200.

The reference package (yiannisha/robotics-batch-invariant-ops 0.2.0,
installed unmodified into baseline/_ref) is loaded under another module name
so that it and this library can run side by side, and both are called with
the same bf16 inputs: matmul_persistent / linear (batch_invariant_ops.py:
61-139, 271-343, 1608-1616), bmm_persistent (:143-229, 346-431), softmax /
log_softmax (:975-1145), SDPA (:1148-1213) and the MoE (moe.py:11-92).

Bar: normwise relative difference <= 1e-2 between the two implementations
and of each against the fp64 oracle (bf16 tolerance of the benchmark
contract).  The reference's Triton kernels cannot run under the CPU
interpreter in bf16 (its tl.dot is wrong there), so this is the only place
bf16 results are compared with the reference itself.  Skipped when the
reference is not installed.  Only this test imports the reference; the
library never does.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest
import torch

import batch_invariant_ops as ours
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "batch_invariant_ops"
BF16 = torch.bfloat16
BAR = 1e-2


def _load_reference():
    if not (REF_DIR / "__init__.py").exists():
        pytest.skip("reference package not installed in baseline/_ref")
    try:
        import triton  # noqa: F401
    except ImportError:
        pytest.skip("triton not importable")
    name = "bio_reference_triton"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, REF_DIR / "__init__.py", submodule_search_locations=[str(REF_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def ref():
    return _load_reference()


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.double().cpu(), b.double().cpu()
    return float((a64 - b64).norm() / b64.norm().clamp_min(1e-300))


def _agree(mine, theirs, oracle, what):
    d_ref = _rel(mine, theirs)
    d_ours = _rel(mine, oracle)
    d_theirs = _rel(theirs, oracle)
    assert d_ref <= BAR, f"{what}: ours vs reference Triton {d_ref:.3e}"
    assert d_ours <= BAR, f"{what}: ours vs fp64 oracle {d_ours:.3e}"
    assert d_theirs <= BAR, f"{what}: reference Triton vs fp64 oracle {d_theirs:.3e}"


def _rn(*shape, gen, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=gen) * scale).to(BF16)


@pytest.mark.parametrize("m,n", [(1, 4096), (37, 11008), (512, 4096), (2048, 16384)])
def test_linear_matches_reference_triton(ref, m, n):
    gen = torch.Generator(device="cuda").manual_seed(50_000 + m)
    x, w, b = _rn(m, 4096, gen=gen), _rn(n, 4096, gen=gen, scale=1 / 64), _rn(n, gen=gen, scale=0.02)
    mine = ours.linear_batch_invariant(x, w, b)
    theirs = ref.linear_batch_invariant(x, w, b)
    rows = torch.arange(min(m, 64))
    _agree(mine[rows], theirs[rows], O.linear(x[rows], w, b), f"linear {m}x{n}")


def test_matmul_persistent_matches_reference_triton(ref):
    gen = torch.Generator(device="cuda").manual_seed(50_100)
    a, b = _rn(300, 1024, gen=gen), _rn(1024, 700, gen=gen, scale=1 / 32)
    bias = _rn(700, gen=gen, scale=0.02)
    _agree(ours.matmul_persistent(a, b, bias), ref.matmul_persistent(a, b, bias),
           O.mm(a, b, bias), "matmul_persistent 300x1024x700")


def test_bmm_matches_reference_triton(ref):
    gen = torch.Generator(device="cuda").manual_seed(50_200)
    a, b = _rn(6, 257, 128, gen=gen), _rn(6, 128, 300, gen=gen, scale=1 / 16)
    _agree(ours.bmm_persistent(a, b), ref.bmm_persistent(a, b), O.bmm(a, b), "bmm 6x257x128x300")


@pytest.mark.parametrize("log", (False, True))
@pytest.mark.parametrize("width", (8, 4096, 257152))
def test_row_softmax_matches_reference_triton(ref, log, width):
    gen = torch.Generator(device="cuda").manual_seed(50_300 + width)
    x = _rn(16 if width > 4096 else 256, width, gen=gen, scale=3.0)
    if log:
        mine, theirs, orc = ours.log_softmax(x, -1), ref.log_softmax(x, -1), O.log_softmax(x, -1)
    else:
        mine, theirs, orc = ours.softmax(x, -1), ref.softmax(x, -1), O.softmax(x, -1)
    _agree(mine, theirs, orc, f"{'log_' if log else ''}softmax width {width}")


@pytest.mark.parametrize("mode", ("full", "causal", "mask"))
def test_sdpa_matches_reference_triton(ref, mode):
    gen = torch.Generator(device="cuda").manual_seed(50_400)
    q = _rn(1, 16, 512, 128, gen=gen)
    k, v = _rn(1, 4, 512, 128, gen=gen), _rn(1, 4, 512, 128, gen=gen)
    mask = (torch.rand(1, 1, 512, 512, device="cuda", generator=gen) > 0.1) if mode == "mask" else None
    kw = dict(attn_mask=mask, is_causal=mode == "causal", enable_gqa=True)
    mine = ours.scaled_dot_product_attention_batch_invariant(q, k, v, **kw)
    theirs = ref.scaled_dot_product_attention_batch_invariant(q, k, v, **kw)
    _agree(mine, theirs, O.sdpa(q, k, v, **kw), f"sdpa {mode}")


def test_moe_matches_reference_triton(ref):
    gen = torch.Generator(device="cuda").manual_seed(50_500)
    t, e, d, i = 64, 8, 512, 1408
    hidden = _rn(t, d, gen=gen)
    gate, up = _rn(e, i, d, gen=gen, scale=0.02), _rn(e, i, d, gen=gen, scale=0.02)
    down = _rn(e, d, i, gen=gen, scale=0.02)
    logits = torch.randn(t, e, device="cuda", generator=gen)
    top, sel = torch.topk(logits, 2)
    w = torch.softmax(top, -1)
    mine = ours.deterministic_token_choice_moe(hidden, w, sel, gate, up, down)
    theirs = ref.deterministic_token_choice_moe(hidden, w, sel, gate, up, down)
    _agree(mine, theirs, O.moe(hidden, w, sel, gate, up, down), "moe T=64 E=8 top-2")
