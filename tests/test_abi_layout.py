"""The ctypes mirrors of the C-ABI parameter structs (hachiue_b200/_lib.py)
against include/hachiue_cuda.h: a C program compiled with gcc against the
header prints every struct's size and every field's offset, which must equal
the ctypes layout.  A mismatch would make the library read a field from the
wrong bytes.  CPU only (no GPU, no library call)."""
import ctypes
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def ctypes_structs():
    from hachiue_b200 import _lib
    return {name: cls for name, cls in vars(_lib).items()
            if name.startswith("hcu_") and isinstance(cls, type) and issubclass(cls, ctypes.Structure)}


def test_every_param_struct_is_mirrored():
    text = open(os.path.join(ROOT, "include", "hachiue_cuda.h")).read()
    declared = set(re.findall(r"}\s*(hcu_[a-z0-9_]+)\s*;", text))
    assert declared == set(ctypes_structs())


def test_sizes_and_offsets_match_the_header(tmp_path):
    structs = ctypes_structs()
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "hachiue_cuda.h"', "int main(void) {"]
    for name, cls in sorted(structs.items()):
        lines.append(f'  printf("{name} %zu\\n", sizeof({name}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{name}.{field} %zu\\n", offsetof({name}, {field}));')
    lines += ["  return 0;", "}"]
    src, exe = tmp_path / "layout.c", tmp_path / "layout"
    src.write_text("\n".join(lines) + "\n")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    c_layout = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                            check=True).stdout.splitlines())
    for name, cls in structs.items():
        assert int(c_layout[name]) == ctypes.sizeof(cls), name
        for field, _ in cls._fields_:
            assert int(c_layout[f"{name}.{field}"]) == getattr(cls, field).offset, (name, field)


def test_constants_match_the_header():
    """Every HCU_* integer constant the Python binding also defines (as X or
    HCU_X) has the header's value: formats, dtypes, options, status codes."""
    from hachiue_b200 import _lib
    text = open(os.path.join(ROOT, "include", "hachiue_cuda.h")).read()
    defines = {name: int(value) for name, value in re.findall(r"#define HCU_([A-Z0-9_]+)\s+(\d+)\b", text)}
    mirrored = 0
    for name, value in defines.items():
        for attr in (name, "HCU_" + name):
            if hasattr(_lib, attr):
                assert getattr(_lib, attr) == value, (attr, getattr(_lib, attr), value)
                mirrored += 1
    assert mirrored >= 20
