"""Failure detection on the GPU without a fault.

Every spin in the library's pipelined kernels is a bounded mbarrier wait.
bio_selftest_bounded_wait runs that exit path on purpose (a consumer that
never releases a stage and waits on a barrier nothing arrives at, with a
1 ms limit): the kernel must give up, raise BIO_DEV_TIMEOUT in the status
word, drain its copies, free its tensor memory and return, and the next
launch on the device must run normally.  Nothing here traps, faults or
hangs: the waits end by construction.  The reference's counterpart is a
trapping device assert (batch_invariant_ops/moe.py:67-74).
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from batch_invariant_ops import _lib, linear_batch_invariant
from oracle import bio_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_raises_status_and_context_stays_usable():
    lib = _lib.load()
    gen = torch.Generator(device="cuda").manual_seed(60_000)
    src = torch.randint(0, 256, (8192,), device="cuda", dtype=torch.uint8, generator=gen)
    out = torch.full((4,), -1, device="cuda", dtype=torch.int32)
    _lib.clear_device_status()
    t0 = time.perf_counter()
    rc = lib.bio_selftest_bounded_wait(ctypes.c_void_p(src.data_ptr()),
                                       ctypes.c_void_p(out.data_ptr()), 1_000_000, 0,
                                       _lib.stream_of(src))
    assert rc == _lib.BIO_OK, _lib.status_message(rc)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert out.tolist() == [1, 1, 1, 1], out.tolist()
    assert _lib.device_status() & _lib.BIO_DEV_TIMEOUT
    assert elapsed < 5.0, f"bounded waits took {elapsed:.2f} s"
    _lib.clear_device_status()
    # the context is intact: a normal launch right after gives correct results
    x = torch.randn(5, 256, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(384, 256, device="cuda", generator=gen) / 16).to(torch.bfloat16)
    y = linear_batch_invariant(x, w)
    torch.testing.assert_close(y.double().cpu(), O.linear(x, w), rtol=2e-2, atol=1e-2)
    assert _lib.device_status() == 0


def test_bounded_wait_selftest_rejects_bad_arguments():
    lib = _lib.load()
    src = torch.zeros(8192, device="cuda", dtype=torch.uint8)
    out = torch.zeros(4, device="cuda", dtype=torch.int32)
    stream = _lib.stream_of(src)
    assert lib.bio_selftest_bounded_wait(None, ctypes.c_void_p(out.data_ptr()), 10**6, 0,
                                         stream) == _lib.BIO_ERR_ARG
    assert lib.bio_selftest_bounded_wait(ctypes.c_void_p(src.data_ptr() + 1),
                                         ctypes.c_void_p(out.data_ptr()), 10**6, 0,
                                         stream) == _lib.BIO_ERR_ALIGN
    assert lib.bio_selftest_bounded_wait(ctypes.c_void_p(src.data_ptr()),
                                         ctypes.c_void_p(out.data_ptr()), 10, 0,
                                         stream) == _lib.BIO_ERR_ARG
