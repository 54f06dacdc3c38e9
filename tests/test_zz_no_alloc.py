"""The convolution entry point that allocates nothing (bio_conv_nd_noalloc).

Some callers cannot allocate device memory while they run -- a real-time
robot control loop that reserves all of its memory before the loop starts
(cudaMalloc can block and synchronise the device mid-cycle), or a C/C++ host
without a caching allocator.  For them the library keeps the convolution's
im2col scratch in one fixed device array.  This file is collected last so
that a failure here never hides the result of any other test; it passes both
alone in a fresh process and after the rest of the suite.

The test calls the entry point through the C ABI (ctypes), twice in a row on
the same buffers, and compares each result with the regular entry point
(conv2d/conv3d_batch_invariant: bio_im2col + the same GEMM with
PyTorch-allocated scratch).  Both run the same arithmetic, so the results
must be identical bit for bit (fp32 included: both take the exact-slice
GEMM); the first sample run alone must also give the bits it gets in the
batch.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from batch_invariant_ops import _conv, _lib, conv2d_batch_invariant, conv3d_batch_invariant

pytestmark = pytest.mark.gpu


def _noalloc(x, w, b, stride, padding, dilation, groups, out):
    nd = w.ndim - 2
    geom = _conv._geom(x.shape[0], x.shape[1], groups, x.shape[2:], w.shape[2:], stride, padding,
                       dilation, out.shape[2:])
    return _lib.load().bio_conv_nd_noalloc(
        _lib.DTYPE_CODE[x.dtype],
        ctypes.c_void_p(x.data_ptr()),
        ctypes.c_void_p(w.data_ptr()),
        ctypes.c_void_p(b.data_ptr() if b is not None else 0),
        ctypes.c_void_p(out.data_ptr()),
        ctypes.byref(geom),
        w.shape[0],
        x.device.index,
        _lib.stream_of(x),
    ), nd


CASES = [
    # SigLIP-style 14x14 patch embedding (patches of 588 columns -> padded)
    ("conv2d", (4, 3, 56, 56), (64, 3, 14, 14), (14, 14), (0, 0), (1, 1), 1, torch.bfloat16),
    # grouped, strided, dilated 3x2 kernel: K = 12 per group (weight packed too)
    ("conv2d", (2, 4, 13, 11), (6, 2, 3, 2), (2, 1), (1, 0), (2, 1), 2, torch.float16),
    # Qwen-style 3-D patch embedding, fp32 (CUDA-core GEMM)
    ("conv3d", (3, 3, 2, 16, 16), (12, 3, 2, 16, 16), (2, 16, 16), (0, 0, 0), (1, 1, 1), 1,
     torch.float32),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[7]}")
def test_noalloc_conv_matches_regular_entry_point_twice(case):
    kind, xs, ws, stride, padding, dilation, groups, dtype = case
    gen = torch.Generator(device="cuda").manual_seed(9100)
    x = torch.randn(*xs, device="cuda", generator=gen).to(dtype)
    w = torch.randn(*ws, device="cuda", generator=gen).to(dtype)
    b = torch.randn(ws[0], device="cuda", generator=gen).to(dtype)
    fn = conv2d_batch_invariant if kind == "conv2d" else conv3d_batch_invariant
    expected = fn(x, w, b, stride, padding, dilation, False, (0,) * len(stride), groups)
    out = torch.empty_like(expected)
    for _ in range(2):
        out.fill_(float("nan"))
        rc, _ = _noalloc(x, w, b, stride, padding, dilation, groups, out)
        assert rc == _lib.BIO_OK, _lib.status_message(rc)
        torch.cuda.synchronize()
        assert torch.equal(out, expected), (
            f"max diff {(out.double() - expected.double()).abs().max().item()}")
    # the first sample alone gives the bits it gets inside the batch
    alone = torch.full_like(expected[:1], float("nan"))
    rc, _ = _noalloc(x[:1].contiguous(), w, b, stride, padding, dilation, groups, alone)
    assert rc == _lib.BIO_OK, _lib.status_message(rc)
    torch.cuda.synchronize()
    assert torch.equal(alone, out[:1])


def test_noalloc_conv_rejects_problems_beyond_the_scratch():
    # B * L * K = 64 * 1024 * 768 bf16 = 96 MiB of patches > 32 MiB
    x = torch.zeros(64, 3, 512, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(8, 3, 16, 16, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(64, 8, 32, 32, device="cuda", dtype=torch.bfloat16)
    rc, _ = _noalloc(x, w, None, (16, 16), (0, 0), (1, 1), 1, out)
    assert rc == _lib.BIO_ERR_SCRATCH
    assert "scratch" in _lib.status_message(rc)
    assert torch.count_nonzero(out) == 0
