"""ctypes binding of ``libbio_sm100.so`` (C ABI in ``include/bio_sm100.h``).

The shared object is built in-tree by ``build.py`` and loaded lazily on the
first operator call, so importing the package works on machines without a
GPU.  There is no fallback: when the library is missing or fails to load every
operator raises ``RuntimeError`` naming the problem.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libbio_sm100.so"

# status codes (include/bio_sm100.h)
BIO_OK = 0
BIO_ERR_SHAPE = 1
BIO_ERR_STRIDE = 2
BIO_ERR_ALIGN = 3
BIO_ERR_DTYPE = 4
BIO_ERR_LAUNCH = 5
BIO_ERR_DRIVER = 6
BIO_ERR_ARG = 7
BIO_ERR_DEVICE = 8
BIO_ERR_SCRATCH = 9
NOALLOC_SCRATCH_BYTES = 32 << 20

BIO_DEV_TIMEOUT = 1
BIO_DEV_INDEX = 2

BIO_GEMM_BIAS_PER_ROW = 1
BIO_GEMM_GATE_GELU_TANH = 2

BIO_NORM_LAYER = 0
BIO_NORM_RMS = 1

BIO_F32 = 0
BIO_F16 = 1
BIO_BF16 = 2

DTYPE_CODE = {torch.float32: BIO_F32, torch.float16: BIO_F16, torch.bfloat16: BIO_BF16}


class GemmArgs(ctypes.Structure):
    """Mirror of ``bio_gemm_args``."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("batch1", ctypes.c_int64),
        ("batch2", ctypes.c_int64),
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("a", ctypes.c_void_p),
        ("a_sm", ctypes.c_int64),
        ("a_sk", ctypes.c_int64),
        ("a_s1", ctypes.c_int64),
        ("a_s2", ctypes.c_int64),
        ("a_div2", ctypes.c_int64),
        ("b", ctypes.c_void_p),
        ("b_sk", ctypes.c_int64),
        ("b_sn", ctypes.c_int64),
        ("b_s1", ctypes.c_int64),
        ("b_s2", ctypes.c_int64),
        ("b_div2", ctypes.c_int64),
        ("c", ctypes.c_void_p),
        ("c_sm", ctypes.c_int64),
        ("c_sn", ctypes.c_int64),
        ("c_s1", ctypes.c_int64),
        ("c_s2", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("bias_s2", ctypes.c_int64),
        ("alpha", ctypes.c_float),
        ("device", ctypes.c_int32),
    ]


# name -> (restype, argtypes); every symbol declared in include/bio_sm100.h
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_P = ctypes.c_void_p
SIGNATURES: dict[str, tuple] = {
    "bio_abi_version": (ctypes.c_int, []),
    "bio_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "bio_sm_count": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "bio_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "bio_clear_device_status": (ctypes.c_int, [ctypes.c_int]),
    "bio_gemm": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _P]),
    "bio_gemm_residual": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _P, _I64, _P]),
    "bio_gemm_tile_config": (ctypes.c_int, [_I64, _I64, _I32]),
    "bio_gemm_tile_for": (
        ctypes.c_int,
        [_I64, _I64, _I64, _I32, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_I32)],
    ),
    "bio_gemm_tiled": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _I32, _I32, _P]),
    "bio_gemm_f32_exact_workspace": (_I64, [ctypes.POINTER(GemmArgs)]),
    "bio_gemm_f32_exact": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _P, _I64, _P]),
    "bio_gemm_segmented": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _P, _P]),
    "bio_gemm_swiglu": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _P, _P, _P]),
    "bio_softmax": (ctypes.c_int, [_I32, _I32, _P, _P, _I64, _I64, _I64, _I32, _I32, _P]),
    "bio_reduce": (ctypes.c_int, [_I32, _I32, _I32, _P, _P, _I64, _I64, _I64, _I32, _P]),
    "bio_norm": (
        ctypes.c_int,
        [_I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, ctypes.c_float, _I32,
         _P],
    ),
    "bio_im2col": (ctypes.c_int, [_I32, _P, _P, _P, _I64, _I32, _P]),
    "bio_depthwise_conv1d": (
        ctypes.c_int,
        [_I32, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _P],
    ),
    "bio_conv_transpose": (ctypes.c_int, [_I32, _P, _P, _P, _P, _P, _I64, _I32, _P]),
    "bio_conv_transpose_scatter": (ctypes.c_int, [_I32, _P, _P, _P, _P, _I64, _I32, _P]),
    "bio_attention": (ctypes.c_int, [_P, _P]),
    "bio_attention_varlen": (ctypes.c_int, [_P, _P]),
    "bio_silu_mul": (ctypes.c_int, [_I32, _P, _P, _P, _I64, _I32, _P]),
    "bio_moe_route_sum": (
        ctypes.c_int,
        [_I32, _P, _I32, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
    ),
    "bio_moe_plan_workspace": (_I64, [_I64, _I64, _I64]),
    "bio_moe_plan": (ctypes.c_int, [_P, _I64, _I64, _I64, _P, _I64, _I32, _P]),
    "bio_moe_gather_rows": (ctypes.c_int, [_I32, _P, _I64, _P, _I64, _I64, _I64, _P, _I32, _P]),
    "bio_moe_route_sum_sorted": (
        ctypes.c_int,
        [_I32, _P, _I32, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
    ),
    "bio_selftest_bounded_wait": (ctypes.c_int, [_P, _P, _I64, _I32, _P]),
    "bio_conv_nd_noalloc": (ctypes.c_int, [_I32, _P, _P, _P, _P, _P, _I64, _I32, _P]),
    "bio_pack_rows": (
        ctypes.c_int,
        [_I32, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I32, _P],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the kernel library with typed signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.exists():
            raise RuntimeError(
                f"batch_invariant_ops: CUDA kernel library not found at {target}; "
                "build it with `python robotics-batch-invariant-ops_b200/build.py`"
            )
        lib = ctypes.CDLL(str(target))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def status_message(status: int) -> str:
    return load().bio_status_string(status).decode()


def check(status: int, what: str) -> None:
    """Raise RuntimeError for a non-zero status returned by the library."""
    if status != BIO_OK:
        raise RuntimeError(f"{what} failed: {status_message(status)} (status {status})")


# Current-stream lookup without building a torch.cuda.Stream object per call
# (the raw handle of the same current stream); the public API otherwise.
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(tensor: torch.Tensor) -> ctypes.c_void_p:
    """The current CUDA stream of ``tensor``'s device, as the C ABI takes it."""
    if _RAW_STREAM is not None:
        return ctypes.c_void_p(_RAW_STREAM(tensor.device.index))
    return ctypes.c_void_p(torch.cuda.current_stream(tensor.device).cuda_stream)


def device_status(device: int | torch.device | None = None) -> int:
    """Device status word (OR of BIO_DEV_* bits); synchronises the device."""
    dev = _device_index(device)
    out = ctypes.c_int(0)
    check(load().bio_device_status(dev, ctypes.byref(out)), "bio_device_status")
    return out.value


def clear_device_status(device: int | torch.device | None = None) -> None:
    check(load().bio_clear_device_status(_device_index(device)), "bio_clear_device_status")


def _device_index(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, torch.device):
        return device.index if device.index is not None else torch.cuda.current_device()
    return int(device)
