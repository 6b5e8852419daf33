"""Compile laguna-raw's own GLSL compute shaders for the CPU -> oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The reference (auryn-macmillan/laguna-raw-halo-strix)
is Rust + Vulkan; neither a Rust toolchain nor a Vulkan driver exists here, so
its shaders cannot run as designed.  Their bodies are, however, nearly plain
C: this script reads each `kernels/<name>.comp` where it lies in the reference
tree, rewrites the GLSL-only declarations in memory, and pipes the result to
g++.  Nothing from the reference is written into this repository; the only
output is `oracle/_ref/libref_shaders.so` (git-ignored).

Rewrites (declarations only; the function bodies are compiled as written):
  * `#version`, `layout(local_size_x = ...) in;` are dropped;
  * `layout(binding = N) ... buffer B { T name[]; };` -> `static T* name;`;
  * `layout(push_constant) uniform P { ... };` -> one static global per member;
  * `void main()` -> `static void shader_main()`;
  * `out T p` parameters -> `T& p`;
  * float literals get an `f` suffix so arithmetic stays in single precision
    as GLSL specifies.
Each shader gets an `extern "C" ref_<name>(void **bindings, const void *push,
uint32_t invocations)` entry that binds the buffers and push block, then runs
invocations 0..invocations-1 (OpenMP over invocations, as on the GPU every
invocation is independent).

Usage: python oracle/build_ref.py [--reference DIR]   (default: $LAGUNA_REFERENCE, else
       a directory named `reference` beside the repository root)
"""
from __future__ import annotations

import argparse
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libref_shaders.so")

# The shaders on the quantized projection path and the kernels interleaved with
# it in the DFlash encoder/decoder.
SHADERS = [
    "proj", "proj_q8_0", "proj_q4k", "rmsnorm", "qk_norm_rope", "activation",
    "add", "gate_mul", "mha_attn", "enc_aux_norm",
]

_BUF = re.compile(
    r"layout\s*\(\s*binding\s*=\s*(\d+)[^)]*\)\s*(?:(?:readonly|writeonly|restrict|coherent)\s+)*"
    r"buffer\s+\w+\s*\{\s*(\w+)\s+(\w+)\s*\[\s*\]\s*;\s*\}\s*;",
    re.S,
)
_PUSH = re.compile(r"layout\s*\(\s*push_constant\s*\)\s*uniform\s+\w+\s*\{([^}]*)\}\s*;", re.S)
_LOCAL = re.compile(r"layout\s*\(\s*local_size_x[^)]*\)\s*in\s*;")
_FLOAT = re.compile(r"(?<![\w.])(\d+\.\d*(?:[eE][-+]?\d+)?|\d+[eE][-+]?\d+|\.\d+(?:[eE][-+]?\d+)?)(?![\w.])")


def translate(name: str, src: str) -> str:
    """Return a C++ translation unit for one shader source."""
    src = "\n".join(l for l in src.splitlines() if not l.strip().startswith("#version"))
    src = _LOCAL.sub("", src)

    bindings = []

    def buf(m):
        idx, ty, var = int(m.group(1)), m.group(2), m.group(3)
        bindings.append((idx, ty, var))
        return f"static {ty}* {var};"

    src = _BUF.sub(buf, src)

    push = []

    def pc(m):
        out = []
        for decl in m.group(1).split(";"):
            decl = decl.strip()
            if not decl:
                continue
            ty, var = decl.split()
            push.append((ty, var))
            out.append(f"static {ty} {var};")
        return "\n".join(out)

    src = _PUSH.sub(pc, src)
    src = re.sub(r"\bvoid\s+main\s*\(\s*\)", "static void shader_main()", src)
    src = re.sub(r"\bout\s+(\w+)\s+(\w+)", r"\1& \2", src)
    src = _FLOAT.sub(lambda m: m.group(1) + "f", src)

    bindings.sort()
    lines = [f'#include "{os.path.join(HERE, "glsl_shim.h")}"', "namespace {", src, "}  // namespace", ""]
    lines.append(f'extern "C" void ref_{name}(void **bindings, const void *push, uint32_t invocations) {{')
    for i, (idx, ty, var) in enumerate(bindings):
        lines.append(f"    {var} = static_cast<{ty}*>(bindings[{i}]);  // binding {idx}")
    off = 0
    for ty, var in push:
        lines.append(f"    std::memcpy(&{var}, static_cast<const char*>(push) + {off}, 4);")
        off += 4
    lines.append("    #pragma omp parallel for schedule(static)")
    lines.append("    for (long long i = 0; i < (long long)invocations; i++) {")
    lines.append("        gl_GlobalInvocationID = uvec3{(uint)i, 0u, 0u};")
    lines.append("        shader_main();")
    lines.append("    }")
    lines.append("}")
    lines.append(f'extern "C" uint32_t ref_{name}_push_bytes(void) {{ return {off}u; }}')
    lines.append(f'extern "C" uint32_t ref_{name}_bindings(void) {{ return {len(bindings)}u; }}')
    return "\n".join(lines) + "\n"


def _default_tree() -> str:
    here = os.path.dirname(os.path.abspath(__file__))
    return os.environ.get("LAGUNA_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(here)), "reference")


def build(reference: str, cxx: str = "g++", verbose: bool = False) -> str:
    kdir = os.path.join(reference, "kernels")
    if not os.path.isdir(kdir):
        raise FileNotFoundError(f"reference shaders not found under {kdir}")
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    for name in SHADERS:
        with open(os.path.join(kdir, name + ".comp")) as f:
            tu = translate(name, f.read())
        obj = os.path.join(OUT_DIR, name + ".o")
        cmd = [cxx, "-x", "c++", "-std=c++17", "-O2", "-fPIC", "-fopenmp", "-ffp-contract=off",
               "-fno-fast-math", "-w", "-c", "-o", obj, "-"]
        r = subprocess.run(cmd, input=tu, text=True, capture_output=True)
        if r.returncode != 0:
            raise RuntimeError(f"compiling {name}.comp failed:\n{r.stderr[-4000:]}")
        objs.append(obj)
    cmd = [cxx, "-shared", "-fopenmp", "-o", LIB] + objs + ["-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"linking {LIB} failed:\n{r.stderr[-4000:]}")
    for o in objs:
        os.remove(o)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--cxx", default="g++")
    a = ap.parse_args()
    try:
        build(a.reference or _default_tree(), a.cxx, verbose=True)
    except Exception as e:  # noqa: BLE001
        print(f"build_ref: {e}", file=sys.stderr)
        sys.exit(1)
