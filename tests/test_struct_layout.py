"""The ctypes mirrors of the C ABI's structs (busfill_b200.SweepOp,
busfill_b200.Tensor, busfill_b200.tp.Gather) against include/busfill.h: a
small C program compiled with the host compiler prints each struct's size
and field offsets, which must equal the ctypes layout (a drift would hand the
library shifted fields)."""
import ctypes
import os
import shutil
import subprocess

import pytest

import busfill_b200 as bf
from busfill_b200 import tp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

STRUCTS = {
    "busfill_sweep_op": (bf.SweepOp, ["w", "w_up", "a", "c", "N", "K", "dep"]),
    "busfill_tensor": (bf.Tensor, ["type", "ne", "nb", "data"]),
    "busfill_gather": (tp.Gather, ["npeers", "col_off", "ldc", "out", "flag", "wait", "wait_gen", "nwait",
                                   "wait_tiles"]),
}


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    d = tmp_path_factory.mktemp("layout")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "busfill.h"', "int main(void) {"]
    for name, (_, fields) in STRUCTS.items():
        lines.append(f'  printf("{name} size %zu\\n", sizeof({name}));')
        for f in fields:
            lines.append(f'  printf("{name} {f} %zu\\n", offsetof({name}, {f}));')
    lines += ["  return 0;", "}"]
    src = d / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = d / "layout"
    subprocess.run([cc, "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    res = {}
    for line in out.splitlines():
        name, key, val = line.split()
        res[(name, key)] = int(val)
    return res


@pytest.mark.parametrize("name", sorted(STRUCTS))
def test_ctypes_mirror_matches_c_layout(c_layout, name):
    cls, fields = STRUCTS[name]
    assert ctypes.sizeof(cls) == c_layout[(name, "size")], name
    for f in fields:
        assert getattr(cls, f).offset == c_layout[(name, f)], (name, f)
