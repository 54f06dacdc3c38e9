"""Per-launch records and NVTX ranges for the library's kernels.

The reference attaches launch metadata to its Triton matmul kernels -- a name
carrying M, N, K and the algorithmic flops and bytes of the call
(``_matmul_launch_metadata``, batch_invariant_ops.py:31-47) -- for its
profiler to pick up.  Here every operator wrapper reports the same facts for
the C-ABI call it makes: inside ``record_launches()`` each call appends a
record ``{"op", "name", "flops<bits>", "bytes"}``, and with ``nvtx=True`` the
call is also wrapped in an NVTX range of that name (visible to Nsight and to
``ncu --nvtx``).  Outside the context nothing is recorded and nothing is
pushed (one thread-local check per call).

    with tracing.record_launches(nvtx=True) as records:
        y = linear_batch_invariant(x, w, b)
    records[0]  # {'op': 'gemm', 'name': 'bio_gemm [M=37, N=4096, K=4096, batch=1]',
                #  'flops16': 1.24e9, 'bytes': ...}
"""

from __future__ import annotations

import contextlib
import threading

import torch

_state = threading.local()


def active() -> bool:
    return getattr(_state, "records", None) is not None


@contextlib.contextmanager
def record_launches(nvtx: bool = False):
    """Collect one record per library call made by this thread; optionally
    wrap each call in an NVTX range.  Yields the list the records go to."""
    prev_records = getattr(_state, "records", None)
    prev_nvtx = getattr(_state, "nvtx", False)
    records: list[dict] = []
    _state.records = records
    _state.nvtx = bool(nvtx)
    try:
        yield records
    finally:
        _state.records = prev_records
        _state.nvtx = prev_nvtx


def note(op: str, name: str, flops: float, nbytes: float, elem_bytes: int) -> bool:
    """Append a record (no-op outside record_launches).  Returns whether an
    NVTX range was pushed (the caller pops it with ``done``)."""
    records = getattr(_state, "records", None)
    if records is None:
        return False
    records.append({"op": op, "name": name, f"flops{8 * elem_bytes}": float(flops),
                    "bytes": float(nbytes)})
    if getattr(_state, "nvtx", False):
        torch.cuda.nvtx.range_push(name)
        return True
    return False


def done(pushed: bool) -> None:
    if pushed:
        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def span(op: str, name: str, flops: float, nbytes: float, elem_bytes: int):
    """``note`` + ``done`` around a block (a no-op outside record_launches)."""
    pushed = note(op, name, flops, nbytes, elem_bytes) if active() else False
    try:
        yield
    finally:
        done(pushed)
