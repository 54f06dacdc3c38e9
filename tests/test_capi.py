"""CPU checks of the C ABI: the library loads without a GPU and exports every
function declared in include/bio_sm100.h; the ctypes signature table matches
the header; the K block that fixes every GEMM element's accumulation order
depends on the dtype only, and the output-tile policy (bio_gemm_tile_for)
returns only tiles that the library builds (which tile runs is a function of
m as well: tests/test_gemm_gpu.py runs every such tile on the same inputs and
requires identical bits)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from batch_invariant_ops import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "bio_sm100.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bio_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "bio_gemm" in names and "bio_abi_version" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"symbols declared but not exported: {missing}"


def test_ctypes_table_matches_header():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert lib.bio_abi_version() == 1
    assert lib.bio_status_string(0).decode() == "ok"
    assert "alignment" in lib.bio_status_string(_lib.BIO_ERR_ALIGN).decode()


def test_gemm_args_struct_layout():
    # 2 int32 + 5 int64 + ptr + 5 int64 + ptr + 5 int64 + ptr + 4 int64 + ptr + int64
    # + float + int32
    assert ctypes.sizeof(_lib.GemmArgs) == 8 + 5 * 8 + 8 + 5 * 8 + 8 + 5 * 8 + 8 + 4 * 8 + 8 + 8 + 8


@pytest.mark.parametrize("dtype", (torch.float32, torch.float16, torch.bfloat16))
@pytest.mark.parametrize("n", (1, 91, 4096, 11008, 16384, 184622))
def test_k_block_is_fixed_by_dtype(n, dtype):
    from batch_invariant_ops import _gemm

    bm, bn, bk = _gemm.tile_config(n, 4096, dtype)
    if dtype == torch.float32:
        assert (bm, bn, bk) == (128, 128, 8)
    else:
        assert bk == 64, "the 16-bit K order is 64-wide blocks for every shape"
        assert bm in (128, 256) and bn in (64, 128, 256)


BUILT_TILES = {(128, 32), (128, 64), (128, 96), (128, 128), (128, 256), (256, 128), (256, 256)}


@pytest.mark.parametrize("n", (8, 64, 65, 1152, 4096, 11008, 16384, 184622))
@pytest.mark.parametrize("b_mn", (False, True))
def test_tile_policy_returns_built_tiles(n, b_mn):
    from batch_invariant_ops import _gemm

    for m in (1, 8, 32, 127, 128, 129, 256, 400, 512, 1152, 2048, 8192, 65536):
        for batch in (1, 3, 64):
            tile = _gemm.tile_for(m, n, batch, 148, b_mn)
            assert tile in BUILT_TILES, (m, n, batch, tile)
            if m <= 128:
                assert tile[0] == 128, "one m-block runs single-CTA tiles"
            if b_mn and tile[0] == 128:
                assert tile[1] in (64, 128, 256), "an N-contiguous B needs whole 64-column atoms"


def test_tile_policy_rejects_bad_arguments():
    lib = _lib.load()
    tm, tn = ctypes.c_int32(0), ctypes.c_int32(0)
    assert lib.bio_gemm_tile_for(0, 8, 1, 148, 0, ctypes.byref(tm), ctypes.byref(tn)) == _lib.BIO_ERR_ARG
    assert lib.bio_gemm_tile_for(8, 8, 1, 0, 0, ctypes.byref(tm), ctypes.byref(tn)) == _lib.BIO_ERR_ARG
    assert lib.bio_gemm_tile_for(8, 8, 1, 148, 0, None, ctypes.byref(tn)) == _lib.BIO_ERR_ARG


def test_gemm_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    args = _lib.GemmArgs()
    args.dtype = 99
    args.batch1 = args.batch2 = 1
    args.m = args.n = args.k = 4
    args.a_div2 = args.b_div2 = 1
    assert lib.bio_gemm(ctypes.byref(args), None) == _lib.BIO_ERR_DTYPE
    args.dtype = _lib.BIO_BF16
    args.flags = 4  # unknown flag bit
    assert lib.bio_gemm(ctypes.byref(args), None) == _lib.BIO_ERR_ARG
    args.flags = 0
    args.batch2 = 0
    assert lib.bio_gemm(ctypes.byref(args), None) == _lib.BIO_ERR_SHAPE
    assert lib.bio_gemm(None, None) == _lib.BIO_ERR_ARG


def test_struct_layouts_match_the_c_header(tmp_path):
    """Compile a C probe against include/bio_sm100.h and compare sizeof/offsets
    of every ABI struct with the ctypes mirrors."""
    import shutil
    import subprocess

    from batch_invariant_ops import _attn, _conv

    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    mirrors = {
        "bio_gemm_args": _lib.GemmArgs,
        "bio_attn_args": _attn._AttnArgs,
        "bio_conv_geom": _conv._Geom,
    }
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){"]
    for cname, py in mirrors.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            cfield = {"inp": "in"}.get(fname, fname)
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {cfield}));')
    lines.append("return 0;}")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run([gcc, str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.splitlines())
    for cname, py in mirrors.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def _noalloc_geom(batch, channels, inp, kernel, out):
    from batch_invariant_ops import _conv

    return _conv._geom(batch, channels, 1, inp, kernel, (1,) * len(inp), (0,) * len(inp),
                       (1,) * len(inp), out)


def test_noalloc_conv_rejects_sizes_that_would_wrap_without_gpu():
    """B * G * L * Kpad * dtype bytes would wrap past 2^64 to a small number;
    the entry point must see the overflow and refuse before touching the GPU
    (none here: a launch would return BIO_ERR_LAUNCH, not BIO_ERR_SCRATCH)."""
    lib = _lib.load()
    geom = _noalloc_geom(2**61, 1, (1, 1), (1, 1), (1, 1))
    dummy = ctypes.c_void_p(256)
    rc = lib.bio_conv_nd_noalloc(_lib.BIO_BF16, dummy, dummy, None, dummy, ctypes.byref(geom), 1,
                                 0, None)
    assert rc == _lib.BIO_ERR_SCRATCH
    geom = _noalloc_geom(1, 2**40, (1, 1), (2**12, 2**12), (1, 1))
    rc = lib.bio_conv_nd_noalloc(_lib.BIO_BF16, dummy, dummy, None, dummy, ctypes.byref(geom), 1,
                                 0, None)
    assert rc in (_lib.BIO_ERR_SCRATCH, _lib.BIO_ERR_SHAPE)


def test_noalloc_conv_rejects_inconsistent_output_extent_without_gpu():
    lib = _lib.load()
    dummy = ctypes.c_void_p(256)
    # a 3x3 input with a 3x3 kernel gives a 1x1 output, not 2x2
    geom = _noalloc_geom(1, 4, (3, 3), (3, 3), (2, 2))
    rc = lib.bio_conv_nd_noalloc(_lib.BIO_BF16, dummy, dummy, None, dummy, ctypes.byref(geom), 8,
                                 0, None)
    assert rc == _lib.BIO_ERR_SHAPE
