"""The ctypes structs of flash_mlm._lib match include/flash_mlm.h byte for byte.

A small C program (compiled here with the host C compiler against the header)
prints sizeof and every field's offsetof for the three argument structs; the
ctypes mirrors must agree, so a field added or reordered on one side only is
caught before any kernel call reads a misplaced pointer.
"""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None and shutil.which("cc") is None, reason="no C compiler")
def test_ctypes_structs_match_header(tmp_path):
    from flash_mlm import _lib

    structs = {"fmlm_view4": _lib.View4, "fmlm_dense_args": _lib.DenseArgs, "fmlm_packed_args": _lib.PackedArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "flash_mlm.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "abi.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "abi"
    cc = shutil.which("gcc") or shutil.which("cc")
    subprocess.run([cc, "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, field, value = line.split()
        got[(cname, field)] = int(value)
    for cname, cls in structs.items():
        assert got[(cname, "sizeof")] == __import__("ctypes").sizeof(cls), f"{cname} size"
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, f"{cname}.{fname} offset"
