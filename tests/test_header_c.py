"""include/gpt2q.h is a plain C header: a C99 program that includes it, takes the address of every
declared function and calls the host-only entry points links against libgpt2q.so and runs
without a GPU (the boundary a cgo / JNI / N-API / ctypes binding sees)."""
import os
import re
import shutil
import subprocess

import pytest

from smelt_b200 import smt

ROOT = os.path.join(os.path.dirname(__file__), "..")
HEADER = os.path.join(ROOT, "include", "gpt2q.h")


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c99_program_uses_the_header(tmp_path):
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    names = sorted(set(re.findall(r"\b(gpt2q_\w+)\s*\(", text)))
    refs = "\n".join(f"    fns[n++] = (void (*)(void))&{n};" for n in names)
    src = f"""
#include <stdio.h>
#include <string.h>
#include "gpt2q.h"
int main(void) {{
    void (*fns[{len(names)}])(void);
    int n = 0;
{refs}
    for (int i = 0; i < n; ++i) if (!fns[i]) return 2;
    uint8_t h[32];
    if (gpt2q_blake3("abc", 3, h) != GPT2Q_OK) return 3;
    for (int i = 0; i < 32; ++i) printf("%02x", h[i]);
    printf("\\n");
    char buf[256];
    if (gpt2q_smt_inspect("/nonexistent.smt", 1, buf, sizeof buf) != GPT2Q_EARG) return 4;
    if (strstr(gpt2q_last_error(NULL), "cannot open") == NULL) return 5;
    uint64_t st = gpt2q_rng_new(7);
    uint32_t b[4];
    gpt2q_rng_below(&st, b, 4, 10);
    for (int i = 0; i < 4; ++i) if (b[i] >= 10) return 6;
    return 0;
}}
"""
    c = tmp_path / "use_header.c"
    c.write_text(src)
    exe = tmp_path / "use_header"
    lib = os.path.join(ROOT, "smelt_b200", "_lib")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(c),
                    "-L", lib, "-lgpt2q", "-Wl,-rpath," + os.path.abspath(lib), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.strip() == smt.blake3(b"abc").hex()


def test_rust_sys_crate_declares_every_function_with_the_header_arity():
    """rust/gpt2q-sys/src/lib.rs binds every function of the header, each with the header's number
    of parameters, and the safe wrapper (rust/gpt2q) calls only functions the sys crate declares."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    c_arity = {}
    for name, params in re.findall(r"\b(gpt2q_\w+)\s*\(([^)]*)\)\s*;", text):
        c_arity[name] = 0 if params.strip() in ("", "void") else params.count(",") + 1
    src = open(os.path.join(ROOT, "rust", "gpt2q-sys", "src", "lib.rs")).read()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    rust_arity = {name: (0 if not params.strip() else params.count(",") + 1)
                  for name, params in re.findall(r"pub fn (gpt2q_\w+)\(([^)]*)\)", block)}
    assert rust_arity == c_arity
    consts = dict(re.findall(r"pub const (GPT2Q_\w+): c_int = (-?\d+);", src))
    for name, value in re.findall(r"#define (GPT2Q_\w+) (-?\d+)", open(HEADER).read()):
        assert consts.get(name) == value, name
    wrapper = open(os.path.join(ROOT, "rust", "gpt2q", "src", "lib.rs")).read()
    used = set(re.findall(r"sys::(gpt2q_\w+)\(", wrapper))
    assert used and used <= set(c_arity), used - set(c_arity)
