"""The C-ABI boundary, checked without a GPU: the library loads, exports every
function include/draftkv_b200.h declares, and the ctypes mirrors of the C
structs have the same size and field offsets as gcc computes from the header."""

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from draftkv import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "draftkv_b200.h"

STRUCTS = {
    "dkv_full_cache": _lib.FullCacheS, "dkv_comp_cache": _lib.CompCacheS, "dkv_dims": _lib.DimsS,
    "dkv_epilogue": _lib.EpilogueS, "dkv_layer": _lib.LayerS, "dkv_model": _lib.ModelS,
    "dkv_step": _lib.StepS,
}


def declared_functions():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"DKV_API\s+[\w\s\*]+?\b(dkv_\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from importlib import import_module
        import_module("build", None) if False else None
        subprocess.run(["python", str(ROOT / "draft-kv_b200" / "build.py")], check=True)
    return _lib.load(require_device=False)


def test_library_exports_every_declared_function(lib):
    names = declared_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (dkv_\w+)", out))
    assert set(names) <= exported, set(names) - exported
    assert set(_lib.exported_symbols()) == set(names)


def test_version_and_error_string(lib):
    assert lib.dkv_version() == 10000
    assert isinstance(lib.dkv_last_error(), bytes)


def test_argument_errors_are_reported_not_faulted(lib):
    # host-side validation rejects bad arguments before any launch
    st = lib.dkv_quantize(None, 4, 64, 4, None, None, None, None, None)
    assert st == _lib.EINVAL
    assert b"bad arguments" in lib.dkv_last_error()
    st = lib.dkv_quantize(C.c_void_p(16), 4, 64, 5, None, None, None, None, None)
    assert st == _lib.EINVAL and b"bits" in lib.dkv_last_error()


def header_struct_fields():
    """Field names of each `typedef struct {...} name;` in the header."""
    txt = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for body, name in re.findall(r"typedef struct\s*\{(.*?)\}\s*(\w+);", txt, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            for part in decl.split(","):
                m = re.search(r"(\w+)\s*$", part.strip())
                if m:
                    fields.append(m.group(1))
        out[name] = fields
    return out


def test_ctypes_mirrors_every_header_field():
    hdr = header_struct_fields()
    assert set(hdr) == set(STRUCTS)
    for cname, cls in STRUCTS.items():
        assert [f for f, _ in cls._fields_] == hdr[cname], cname


def test_struct_layouts_match_the_header(tmp_path):
    prog = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for cname, cls in STRUCTS.items():
        prog.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            prog.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    prog.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(prog))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.rsplit(" ", 1) for l in lines if l)
    for cname, cls in STRUCTS.items():
        assert int(got[f"{cname} size"]) == C.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(cls, fname).offset, f"{cname}.{fname}"
