"""C ABI checks that need no GPU: the library loads, exports every entry point that
include/actrain.h declares, and the ctypes mirror lays structs out like the C compiler."""
import ctypes as C
import os
import re
import subprocess

import pytest

import actrain as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "actrain.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(act_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(A.LIB_PATH)
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n


def test_binding_covers_header():
    assert set(declared()) == set(A.SIGNATURES)


def test_struct_layouts_match_c(tmp_path):
    src = tmp_path / "layout.c"
    structs = {"act_model_desc": A.ModelDesc, "act_adapter_desc": A.AdapterDesc,
               "act_mf_batch": A.MfBatch, "act_mg_batch": A.MgBatch, "act_opt": A.Opt}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "actrain.h"', "int main(void){"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I" + os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in out if l.strip())
    for cname, py in structs.items():
        assert int(got[cname]) == C.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, (cname, f)


def test_create_reports_errors_without_throwing():
    # Invalid configuration is rejected before any device work.
    md = A.mf_model(100, 4, 2, 256)  # dim != heads * 64 handled as head_dim 50 -> rejected
    ad = A.AdapterDesc(A.ADAPTER_LORA, 4, 8.0, 0, 0x1F, 0, 1, 10, 8, 0)
    with pytest.raises(A.ActError) as e:
        A.Context(md, ad)
    assert e.value.code == A.ACT_ERR_INVALID
