"""The ctypes mirrors of the C-ABI structs (zero_b200/_lib.py) against the
structs as a C compiler lays them out from include/zgpu.h: every struct's
size and every field's offset must agree, so that a field added on one side
only (an ABI drift) fails here on the CPU rather than as wrong values on a GPU.
"""
import ctypes as C
import shutil
import subprocess
from pathlib import Path

import pytest

from zero_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
MIRRORS = {
    "zgpu_opts": _lib.ZgpuOpts,
    "zgpu_qwen3_layer": _lib.ZgpuQwen3Layer,
    "zgpu_qwen3_desc": _lib.ZgpuQwen3Desc,
    "zgpu_ds2_layer": _lib.ZgpuDs2Layer,
    "zgpu_ds2_desc": _lib.ZgpuDs2Desc,
    "zgpu_perf": _lib.ZgpuPerf,
    "zgpu_smodel_info": _lib.ZgpuSmodelInfo,
    "zgpu_smodel_tensor": _lib.ZgpuSmodelTensor,
}


def c_layout(tmp_path):
    """{struct: (size, {field: offset})} printed by a program built against zgpu.h."""
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "zgpu.h"', "int main(void) {"]
    for name, mirror in MIRRORS.items():
        lines.append(f'  printf("%s size %zu\\n", "{name}", sizeof({name}));')
        for field, *_ in mirror._fields_:
            lines.append(f'  printf("%s %s %zu\\n", "{name}", "{field}", offsetof({name}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    out: dict = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        name, key, val = line.split()
        size, fields = out.setdefault(name, [None, {}])
        if key == "size":
            out[name][0] = int(val)
        else:
            fields[key] = int(val)
    return out


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_ctypes_mirrors_match_the_header(tmp_path):
    layout = c_layout(tmp_path)
    for name, mirror in MIRRORS.items():
        size, fields = layout[name]
        assert C.sizeof(mirror) == size, (name, C.sizeof(mirror), size)
        for field, *_ in mirror._fields_:
            assert getattr(mirror, field).offset == fields[field], (name, field)
