"""CPU: the ctypes mirrors of the ABI's structures have exactly the C layout
of include/acefa.h (size and every field offset), checked against a C program
compiled from the header with gcc."""
import ctypes
import os
import shutil
import subprocess

import pytest

import acefa

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

STRUCTS = {
    "acefa_tensor": (acefa.Tensor, ["type", "ne", "nb", "data"]),
    "acefa_mask_gen": (acefa.MaskGen, ["kind", "window", "pos0", "len"]),
    "acefa_rope_norm": (acefa.RopeNormC, ["norm_weight", "eps", "theta_base", "positions"]),
    "acefa_op_ext": (acefa.OpExt, ["mask_gen", "q_prologue", "k_new", "v_new", "append_pos", "k_prologue",
                                   "mirrors", "n_mirrors"]),
}


def _c_layout():
    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    out_dir = os.path.join(HERE, "cpp", "_build")
    os.makedirs(out_dir, exist_ok=True)
    src = os.path.join(out_dir, "layout.c")
    exe = os.path.join(out_dir, "layout")
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "acefa.h"', "int main(void) {"]
    for name, (_, fields) in STRUCTS.items():
        lines.append(f'    printf("{name} size %zu\\n", sizeof({name}));')
        for f in fields:
            lines.append(f'    printf("{name} {f} %zu\\n", offsetof({name}, {f}));')
    lines += ["    return 0;", "}"]
    open(src, "w").write("\n".join(lines) + "\n")
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
    res = {}
    for line in subprocess.run([exe], check=True, capture_output=True, text=True).stdout.splitlines():
        name, key, val = line.split()
        res[(name, key)] = int(val)
    return res


def test_ctypes_structures_match_the_header():
    c = _c_layout()
    for name, (cls, fields) in STRUCTS.items():
        assert ctypes.sizeof(cls) == c[(name, "size")], name
        for f in fields:
            assert getattr(cls, f).offset == c[(name, f)], (name, f)
