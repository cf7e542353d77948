"""The C-ABI library loads on a machine without a GPU and exports every declared symbol."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from miniserve_b200 import _capi
from miniserve_b200.build import LIB, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "msattn.h"


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    build()
    return _capi.load()


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"MS_API\s+[\w\s\*]+?\b(ms_\w+)\s*\(", text)


def test_header_declares_what_the_binding_binds() -> None:
    assert sorted(declared_symbols()) == sorted(_capi.EXPORTED)


def test_library_exports_every_declared_symbol(lib: ctypes.CDLL) -> None:
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_only_declared_symbols_are_exported(lib: ctypes.CDLL) -> None:
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert {s for s in exported if s.startswith("ms_")} == set(declared_symbols())


def test_version_and_error_string(lib: ctypes.CDLL) -> None:
    assert lib.ms_version() // 100 == 1
    assert isinstance(lib.ms_last_error(), bytes)


def test_abi_struct_size_matches_header() -> None:
    # 12 int32 + 3 int64 + 8 int32 = 48 + 24 + 32 = 104 bytes
    assert ctypes.sizeof(_capi.MsPlanInfo) == 104


def test_abi_struct_layout_matches_header(tmp_path: Path) -> None:
    """Every MsPlanInfo field sits at the same offset (and the struct has the same size) in the
    C header as in the ctypes binding: a C program compiled against the header prints them."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    names = [name for name, _ in _capi.MsPlanInfo._fields_]
    src = ["#include <stddef.h>", "#include <stdio.h>", f'#include "{HEADER}"', "int main(void) {",
           '  printf("size %zu\\n", sizeof(MsPlanInfo));']
    src += [f'  printf("{n} %zu\\n", offsetof(MsPlanInfo, {n}));' for n in names]
    src += ["  return 0;", "}"]
    (tmp_path / "layout.c").write_text("\n".join(src) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", "-o", str(exe), str(tmp_path / "layout.c")], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    assert int(got.pop("size")) == ctypes.sizeof(_capi.MsPlanInfo)
    for n in names:
        assert int(got[n]) == getattr(_capi.MsPlanInfo, n).offset, n


def test_calls_reject_bad_arguments_without_touching_a_gpu(lib: ctypes.CDLL) -> None:
    # Argument validation happens before any CUDA call.
    rc = lib.ms_paged_attention(None, 0, None, 0, 16, 8, None, None, 0, None, None, None, 0,
                                1.0, None)
    assert rc == _capi.MS_ERR_ARG
    rc = lib.ms_qk_norm_rope_scatter(None, 0, 4, 15, 8, None, None, 1e-6, None, None, 0, None, 0,
                                     None, None, 0, None, None, 0, None)
    assert rc == _capi.MS_ERR_ARG
    assert b"num_heads" in lib.ms_last_error()
