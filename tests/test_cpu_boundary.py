"""The drop-in boundary as a Rust caller would bind it, checked without a Rust toolchain: every
`fn vg_*` in the `extern "C"` blocks that INTEGRATION.md gives the reference-side maintainer
matches include/voxgen_cuda.h parameter by parameter (C types mapped to their Rust FFI
spellings, pointer constness included), every `#[repr(C)]` struct there matches the header's
struct field by field, and the header compiles as plain C99."""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "voxgen_cuda.h"
INTEGRATION = ROOT / "INTEGRATION.md"

SCALARS = {"int": "c_int", "uint32_t": "u32", "int32_t": "i32", "uint64_t": "u64", "int64_t": "i64", "uint16_t": "u16",
           "uint8_t": "u8", "size_t": "usize",
           "float": "f32", "double": "f64", "char": "c_char", "void": "c_void"}


def rust_name(c_name: str) -> str:
    if c_name in SCALARS:
        return SCALARS[c_name]
    assert c_name.startswith("vg_"), c_name
    return "Vg" + "".join(w.capitalize() for w in c_name[3:].split("_"))


def c_to_rust(ctype: str) -> str:
    """`const float **` -> `*mut *const f32`: each `*` is a Rust pointer whose mutability is the
    constness of what it points to."""
    toks = re.findall(r"\w+|\*", ctype)
    quals, base, cur = [], None, False
    for t in toks:
        if t == "const":
            cur = True
        elif t == "*":
            quals.append(cur)
            cur = False
        else:
            base = t
    # quals[i] is the constness of the object pointer i+1 points to
    out = rust_name(base)
    for q in quals:
        out = f"*{'const' if q else 'mut'} {out}"
    return out


def norm(t: str) -> str:
    return re.sub(r"\s+", " ", t.strip())


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"^(int|const char \*)\s*(vg_\w+)\(([^;]*?)\);", text, flags=re.M | re.S):
        ret, name, params = m.groups()
        ps = [] if params.strip() in ("", "void") else [p.strip() for p in params.split(",")]
        types = []
        for p in ps:
            ident = re.findall(r"\w+", p)[-1]   # the parameter name
            types.append(norm(c_to_rust(p[: p.rfind(ident)])))
        out[name] = (norm(c_to_rust(ret)), types)
    return out


def header_structs():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for m in re.finditer(r"typedef struct (vg_\w+) \{(.*?)\} \1;", text, flags=re.S):
        fields = []
        for decl in m.group(2).split(";"):
            decl = decl.strip()
            if not decl:
                continue
            arr = re.match(r"(.*?)(\w+)\s*\[(\d+)\]$", decl)   # char name[24] -> [c_char; 24]
            if arr:
                fields.append((arr.group(2), f"[{c_to_rust(arr.group(1))}; {arr.group(3)}]"))
                continue
            ident = re.findall(r"\w+", decl)[-1]
            fields.append((ident, norm(c_to_rust(decl[: decl.rfind(ident)]))))
        out[rust_name(m.group(1))] = fields
    return out


def rust_blocks():
    return re.findall(r"```rust\n(.*?)```", INTEGRATION.read_text(), flags=re.S)


def rust_functions():
    out = {}
    for block in rust_blocks():
        for m in re.finditer(r"fn (vg_\w+)\((.*?)\)\s*->\s*([^;]+);", block, flags=re.S):
            name, params, ret = m.groups()
            types = [norm(p.split(":", 1)[1]) for p in params.split(",") if p.strip()]
            out.setdefault(name, []).append((norm(ret), types))
    return out


def rust_structs():
    out = {}
    for block in rust_blocks():
        for m in re.finditer(r"pub struct (Vg\w+)\s*\{(.*?)\}", block, flags=re.S):
            fields = []
            for f in m.group(2).split(","):
                f = f.strip()
                if f:
                    name, ty = f.replace("pub ", "", 1).split(":", 1)
                    fields.append((name.strip(), norm(ty)))
            out[m.group(1)] = fields
    return out


def test_rust_externs_match_the_header():
    hdr = header_functions()
    rs = rust_functions()
    assert len(rs) >= 20, "INTEGRATION.md lost its extern blocks"
    for name, decls in rs.items():
        assert name in hdr, f"{name} is bound in INTEGRATION.md but not declared in the header"
        for ret, types in decls:
            assert (ret, types) == hdr[name], f"{name}: Rust {ret} {types} vs header {hdr[name]}"


def test_rust_structs_match_the_header():
    hdr = header_structs()
    rs = rust_structs()
    assert rs, "INTEGRATION.md lost its #[repr(C)] structs"
    text = HEADER.read_text()
    opaque = {rust_name(n) for n in re.findall(r"typedef struct (vg_\w+) \1;", text)}
    assert opaque == {"VgCtx", "VgModel", "VgStream"}, opaque
    for name, fields in rs.items():
        if fields == [("_p", "[u8; 0]")]:   # an opaque handle type
            assert name in opaque, f"{name} is opaque in INTEGRATION.md but not in the header"
            continue
        assert name in hdr, f"{name} is defined in INTEGRATION.md but not in the header"
        assert fields == hdr[name], f"{name}: Rust {fields} vs header {hdr[name]}"


def test_type_mapping_examples():
    assert c_to_rust("const float **") == "*mut *const f32"
    assert c_to_rust("vg_stream *const *") == "*const *mut VgStream"
    assert c_to_rust("vg_ctx **") == "*mut *mut VgCtx"
    assert c_to_rust("const char *") == "*const c_char"
    assert c_to_rust("uint32_t") == "u32"


def test_header_compiles_as_c99(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "use_header.c"
    src.write_text('#include "voxgen_cuda.h"\nint main(void) { return 0; }\n')
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-fsyntax-only",
                        "-I", str(ROOT / "include"), str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_rust_examples_call_only_declared_functions():
    declared = set(rust_functions())
    called = {m.group(1) for b in rust_blocks() for m in re.finditer(r"(?<!fn )\b(vg_\w+)\(", b)}
    assert called <= declared, sorted(called - declared)
