"""Builds oracle/_ref/libvoxgen_ref.so: VoxGen's own BaseLM compute shaders, read where they lie
in the reference checkout (shaders/*.comp), compiled by g++ as C++ and run on the CPU by the
workgroup emulator in workgroup.cpp.

TEST INFRASTRUCTURE ONLY: the library pins the oracle's restatement against the reference's own
shader code. Nothing in the product links it, and the GPU box never rebuilds it.

The shader bodies compile unchanged against glsl_shim.h. Only the declarations that are GLSL
syntax, not C++, are rewritten, mechanically, into a temporary file that is deleted after the
build (no reference source is written into the repository):
  - `#version` is dropped;
  - `layout(local_size_x = N) in;` becomes a constant;
  - each `layout(..., binding = B) buffer Name { T member[]; } inst;` becomes a struct holding a
    pointer, bound from the dispatch's buffer list at index B;
  - `layout(push_constant) uniform Push {` becomes `struct Push {` (its members are 32-bit
    scalars, so the C++ layout equals the std430 push-constant layout);
  - `void main()` becomes `void vgref_main()` inside a namespace per shader.
Unsuffixed floating constants are single precision (-fsingle-precision-constant), as in GLSL, and
multiply-adds are not contracted (-ffp-contract=off).

Exported per shader S: int vgref_dispatch_S(void *const *buffers, uint32_t n_buffers,
const void *push, uint32_t push_bytes, uint32_t gx, uint32_t gy, uint32_t gz), which returns 0,
-1 for a wrong buffer count, -2 for a wrong push-constant size.
"""
import os
import re
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE = HERE.parent
OUT_DIR = ORACLE / "_ref"
LIB = OUT_DIR / "libvoxgen_ref.so"
# The VoxGen checkout: $VOXGEN_REFERENCE, else a directory named "reference" beside this
# repository's root (the layout the build machine uses).
DEFAULT_REFERENCE = ORACLE.parent.parent / "reference"

# The normal (non-_xtx7900) shaders that BaseLM's decode step records (baselm.rs:892-1052),
# and the three ResidualLM adds around the same layers (acoustic.rs:921-966): FSQ's linear
# layers with bias, its quantiser, and the fusion projection.
SHADERS = ["embedding", "rmsnorm", "residual_rmsnorm", "qkv_matvec", "rope", "store_kv",
           "attn_scores", "softmax", "attn_values", "matvec", "matvec_swiglu",
           "linear_bias", "fsq_quantize", "fusion_linear"]
# The RX 7900 XTX mode swaps these for their _xtx7900 variants (GpuContext::select_spirv at
# baselm.rs:515-546 and :1241): the same bindings and push constants, wave32 subgroup reductions.
XTX_SHADERS = ["rmsnorm", "residual_rmsnorm", "qkv_matvec", "matvec_swiglu", "matvec",
               "attn_scores", "softmax"]
SHADERS += [f"{s}_xtx7900" for s in XTX_SHADERS]

_BUF = re.compile(r"layout\s*\(([^)]*)\)\s*((?:(?:readonly|writeonly|coherent|restrict|volatile)\s+)*)"
                  r"buffer\s+(\w+)\s*\{\s*(\w+)\s+(\w+)\s*\[\s*\]\s*;\s*\}\s*(\w+)\s*;")
_LOCAL = re.compile(r"layout\s*\(\s*local_size_x\s*=\s*(\d+)\s*\)\s*in\s*;")
_PUSH = re.compile(r"layout\s*\(\s*push_constant\s*\)\s*uniform\s+(\w+)\s*\{")
_PUSH_INST = re.compile(r"struct\s+(\w+)\s*\{[^}]*\}\s*(\w+)\s*;")


def reference_dir():
    return Path(os.environ.get("VOXGEN_REFERENCE", DEFAULT_REFERENCE))


def translate(name: str, src: str) -> str:
    """C++ for one shader: the rewritten declarations and the unchanged body in namespace
    vgref_<name>, plus its exported dispatch function."""
    text = re.sub(r"^\s*#version[^\n]*\n", "", src, flags=re.M)
    text = re.sub(r"^\s*#extension[^\n]*\n", "", text, flags=re.M)
    m = _LOCAL.search(text)
    if not m:
        raise ValueError(f"{name}: no local_size_x")
    local = int(m.group(1))
    text = _LOCAL.sub(f"static const uint vgref_local_size = {local}u;", text)
    bindings = []

    def buf(mm):
        quals = mm.group(1)
        b = re.search(r"binding\s*=\s*(\d+)", quals)
        if not b:
            raise ValueError(f"{name}: buffer {mm.group(3)} without binding")
        bindings.append((int(b.group(1)), mm.group(6), mm.group(5), mm.group(4)))
        return f"struct {mm.group(3)} {{ {mm.group(4)} *{mm.group(5)}; }}; static {mm.group(3)} {mm.group(6)};"

    text = _BUF.sub(buf, text)
    if re.search(r"\bbuffer\s+\w+\s*\{", text):
        raise ValueError(f"{name}: a buffer declaration was not recognised")
    text = _PUSH.sub(r"struct \1 {", text)
    pm = _PUSH_INST.search(text[text.find("struct Push"):]) if "struct Push" in text else None
    push_inst = pm.group(2) if pm else None
    text = re.sub(r"\bvoid\s+main\s*\(\s*\)", "void vgref_main()", text)
    bindings.sort()
    if [b[0] for b in bindings] != list(range(len(bindings))):
        raise ValueError(f"{name}: bindings are not 0..n-1")
    bind_lines = "\n".join(f"  {inst}.{member} = ({typ} *)b[{i}];" for i, inst, member, typ in bindings)
    push_size = f"sizeof({push_inst})" if push_inst else "0"
    push_copy = f"  __builtin_memcpy(&{push_inst}, push, sizeof({push_inst}));" if push_inst else ""
    return f"""#include "glsl_shim.h"
namespace vgref_{name} {{
{text}
}}  // namespace vgref_{name}
extern "C" int vgref_dispatch_{name}(void *const *b, uint32_t nb, const void *push, uint32_t push_bytes,
                                     uint32_t gx, uint32_t gy, uint32_t gz) {{
  using namespace vgref_{name};
  if (nb != {len(bindings)}u) return -1;
  if (push_bytes != {push_size}) return -2;
{bind_lines}
{push_copy}
  return vgref::dispatch(&vgref_main, vgref_local_size, gx, gy, gz);
}}
"""


def build(reference=None, force=False, quiet=True) -> Path:
    ref = Path(reference) if reference else reference_dir()
    shaders = ref / "shaders"
    if not shaders.is_dir():
        raise FileNotFoundError(f"reference shaders not found under {ref}")
    deps = [shaders / f"{s}.comp" for s in SHADERS] + [HERE / "glsl_shim.h", HERE / "workgroup.h",
                                                       HERE / "workgroup.cpp", Path(__file__)]
    if LIB.exists() and not force and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix="voxgen_ref_"))
    try:
        srcs = []
        for s in SHADERS:
            cpp = tmp / f"{s}.cpp"
            cpp.write_text(translate(s, (shaders / f"{s}.comp").read_text()))
            srcs.append(str(cpp))
        out = tmp / LIB.name
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp", "-fsingle-precision-constant",
               "-ffp-contract=off", "-fno-fast-math", "-Wno-unused-function", f"-I{HERE}",
               *srcs, str(HERE / "workgroup.cpp"), "-o", str(out)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("g++ failed:\n" + r.stderr[-4000:])
        shutil.move(str(out), str(LIB))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    if not quiet:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(sys.argv[1] if len(sys.argv) > 1 else None, force=True, quiet=False)
