"""CPU checks of the C ABI: the library loads without a GPU and exports every
function declared in include/bio_sm100.h; the ctypes signature table matches
the header; the GEMM tile choice depends on (N, K, dtype) only."""

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
def test_tile_config_is_a_function_of_n_k_dtype(n, dtype):
    from batch_invariant_ops import _gemm

    cfg = _gemm.tile_config(n, 4096, dtype)
    assert cfg == _gemm.tile_config(n, 4096, dtype)
    bm, bn, bk = cfg
    if dtype == torch.float32:
        assert (bm, bn, bk) == (128, 128, 8)
    else:
        assert bm in (128, 256) and bn in (64, 128, 256) and bk == 64


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
