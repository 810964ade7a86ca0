"""The C ABI's structs as the Python binding lays them out.

Every `typedef struct name { ... } name;` in include/qora_cuda.h is compiled
with gcc into a probe that prints its size and each field's offset and size;
the ctypes mirror in qora_b200/_lib.py must declare the same fields in the
same order at the same offsets, with the same array lengths; so must the
#[repr(C)] structs of the Rust binding (include/qora_cuda_ffi.rs), field by
field in type.  A struct added to the header without a mirror fails here
too.  CPU only (gcc)."""
import ctypes as C
import os
import re
import subprocess
from collections import namedtuple

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qora_cuda.h")

MIRRORS = {
    "qora_q4_host": "Q4Host",
    "qora_layer_host": "LayerHost",
    "qora_talker_host": "TalkerHost",
    "qora_predictor_host": "PredictorHost",
    "qora_text_proj_host": "TextProjHost",
    "qora_prompt_row": "PromptRow",
    "qora_sample_params": "SampleParams",
    "qora_decoder_dims": "DecoderDims",
}


Field = namedtuple("Field", "name n type ptr")


def header_structs():
    """[(struct name, [Field(name, array length or None, C type, is pointer)]), ...]
    in header order."""
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = []
    for m in re.finditer(r"typedef struct (\w+) \{(.*?)\} \1;", src, re.S):
        fields = []
        for decl in m.group(2).split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            t = re.match(r"(?:const )?(\w+) (.*)", decl)
            assert t, decl
            for d in t.group(2).split(","):
                f = re.fullmatch(r"\s*(\**)\s*(\w+)\s*(?:\[(\d+)\])?\s*", d)
                assert f, (m.group(1), d)
                fields.append(Field(f.group(2), int(f.group(3)) if f.group(3) else None, t.group(1),
                                    bool(f.group(1))))
        out.append((m.group(1), fields))
    return out


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    """{struct: (sizeof, {field: (offset, size)})} from gcc."""
    structs = header_structs()
    lines = ['#include "qora_cuda.h"', "#include <stdio.h>", "#include <stddef.h>", "int main(void) {"]
    for s, fields in structs:
        lines.append(f'    printf("S {s} %zu\\n", sizeof({s}));')
        for f in fields:
            f = f.name
            lines.append(f'    printf("F {s} {f} %zu %zu\\n", offsetof({s}, {f}), sizeof((({s} *)0)->{f}));')
    lines += ["    return 0;", "}"]
    d = tmp_path_factory.mktemp("abi")
    src, exe = d / "probe.c", d / "probe"
    src.write_text("\n".join(lines) + "\n")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    lay = {}
    for line in out.splitlines():
        p = line.split()
        if p[0] == "S":
            lay[p[1]] = (int(p[2]), {})
        else:
            lay[p[1]][1][p[2]] = (int(p[3]), int(p[4]))
    return lay


def test_every_header_struct_has_a_mirror():
    names = [s for s, _ in header_structs()]
    assert len(names) >= 8
    assert sorted(names) == sorted(MIRRORS)


@pytest.mark.parametrize("struct", sorted(MIRRORS))
def test_mirror_matches_c_layout(struct, c_layout):
    from qora_b200 import _lib
    cls = getattr(_lib, MIRRORS[struct])
    fields = dict(header_structs())[struct]
    size, offsets = c_layout[struct]
    assert [f for f, _ in cls._fields_] == [f.name for f in fields], struct
    assert C.sizeof(cls) == size, struct
    for f, (_, ctype) in zip(fields, cls._fields_):
        desc = getattr(cls, f.name)
        assert (desc.offset, desc.size) == offsets[f.name], (struct, f.name)
        if f.n is not None:
            assert getattr(ctype, "_length_", None) == f.n, (struct, f.name)


_RUST = {"i32": "int32_t", "i64": "int64_t", "u8": "uint8_t", "u16": "uint16_t", "u32": "uint32_t",
         "f32": "float", "f64": "double"}


def rust_structs():
    """{struct: [Field]} from the binding's #[repr(C)] structs with fields."""
    src = re.sub(r"//[^\n]*", "", open(os.path.join(ROOT, "include", "qora_cuda_ffi.rs")).read())
    out = {}
    for m in re.finditer(r"pub struct (\w+) \{([^}]*)\}", src):
        if re.fullmatch(r"\s*_p:\s*\[u8;\s*0\]\s*", m.group(2)):
            continue  # opaque handle
        fields = []
        for name, ty in re.findall(r"pub (\w+):\s*([^,]+?)\s*(?:,|$)", m.group(2).strip()):
            ptr = ty.startswith("*const") or ty.startswith("*mut")
            ty = re.sub(r"^\*(const|mut)\s+", "", ty)
            arr = re.fullmatch(r"\[(\w+);\s*(\d+)\]", ty)
            n = int(arr.group(2)) if arr else None
            base = arr.group(1) if arr else ty
            fields.append(Field(name, n, _RUST.get(base, base), ptr))
        out[m.group(1)] = fields
    return out


def test_rust_binding_structs_match_header():
    rs = rust_structs()
    hs = dict(header_structs())
    assert sorted(rs) == sorted(hs)
    for s, fields in hs.items():
        assert rs[s] == fields, s
