"""The C ABI as the reference engine would bind it (CPU only).

* include/rustane_cuda.h compiles as plain C99 (gcc -std=c99 -Wall -Werror),
  and a C program linked against librustane_cuda.so calls the host-side entry
  points (rt_learning_rate, rt_lcg_fill, rt_tp_shard) and gets the same values
  as the ctypes binding the tests use.
* crates/cuda-bridge/src/lib.rs (the Rust `extern "C"` block that replaces
  crates/ane-bridge/src/lib.rs:1-9) declares every function of the header,
  with the same argument names and C-compatible types, and nothing else.
  There is no Rust toolchain in this image, so the crate itself is not built.
"""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "rustane_cuda.h"
RUST = ROOT / "crates" / "cuda-bridge" / "src" / "lib.rs"


def header_decls() -> dict[str, tuple[str, list[tuple[str, str]]]]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for d in re.findall(r"RT_API\s+([^;#]+?\));", text, flags=re.S):
        d = " ".join(d.split())
        ret, name, args = re.match(r"(.+?)\s*\b(rt_\w+)\((.*)\)$", d).groups()
        params = []
        for a in [x.strip() for x in args.split(",") if x.strip()]:
            t, n = re.match(r"(.+?)\s*\b(\w+)$", a).groups()
            params.append((t.strip(), n))
        out[name] = (ret.strip(), params)
    return out


_C2RUST = {"int": "c_int", "int32_t": "i32", "int64_t": "i64", "uint32_t": "u32", "uint64_t": "u64",
           "uint8_t": "u8", "float": "f32", "double": "f64", "char": "c_char", "void": "c_void"}


def rust_type(c: str) -> str:
    const = c.startswith("const ")
    base = c[6:] if const else c
    stars = base.count("*")
    base = base.replace("*", "").strip()
    t = _C2RUST.get(base, base)
    for i in range(stars):
        t = ("*const " if i == 0 and const else "*mut ") + t
    return t


def rust_decls() -> dict[str, tuple[str, list[tuple[str, str]]]]:
    text = RUST.read_text()
    block = text[text.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    out = {}
    for name, args, ret in re.findall(r"pub fn (rt_\w+)\(([^)]*)\)\s*(?:->\s*([^;]+))?;", block):
        params = [tuple(x.strip() for x in a.split(":", 1)) for a in args.split(",") if a.strip()]
        out[name] = ((ret or "c_void").strip(), [(t, n) for n, t in params])
    return out


def test_rust_bridge_declares_every_header_function():
    h, r = header_decls(), rust_decls()
    assert len(h) > 40
    assert sorted(h) == sorted(r)
    for name, (ret, params) in h.items():
        r_ret, r_params = r[name]
        assert r_ret == rust_type(ret), name
        assert [n for _, n in params] == [n for _, n in r_params], name
        assert [rust_type(t) for t, _ in params] == [t for t, _ in r_params], name


C_PROGRAM = r"""
#include <stdio.h>
#include "rustane_cuda.h"

int main(void) {
  rt_train_config tc = {3e-4f, 0.1f, 100u, 10000u, 0.9f, 0.95f, 1e-8f, 0.1f, 0.05f, 5.0f, 256.0f, 10u, 1.0f, 0.0f};
  float v[8];
  int head0, heads_loc, hid0, hid_loc, k;
  const uint32_t steps[4] = {0u, 50u, 5000u, 9999u};
  for (k = 0; k < 4; ++k) printf("lr %u %.9e\n", steps[k], (double)rt_learning_rate(steps[k], &tc));
  if (rt_lcg_fill(v, 8, 0.5f) != RT_OK) return 2;
  for (k = 0; k < 8; ++k) printf("lcg %d %.9e\n", k, (double)v[k]);
  for (k = 0; k < 8; ++k) {
    if (rt_tp_shard(52, 17920, 8, k, &head0, &heads_loc, &hid0, &hid_loc) != RT_OK) return 3;
    printf("tp %d %d %d %d %d\n", k, head0, heads_loc, hid0, hid_loc);
  }
  if (rt_tp_shard(4, 256, 8, 0, &head0, &heads_loc, &hid0, &hid_loc) != RT_ERR_SHAPE) return 4;
  if (rt_ctx_create(NULL, 0, 1, RT_CTX_TRAIN, NULL) != RT_ERR_ARG) return 5;
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_compiles_as_c99_and_links(tmp_path):
    from rustane_b200 import TrainConfig, _lib, engine
    lib_path = Path(_lib.lib()._name)
    src = tmp_path / "abi.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(ROOT / "include"),
                    str(src), "-o", str(exe), str(lib_path), f"-Wl,-rpath,{lib_path.parent}"], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, (res.returncode, res.stderr)
    lines = res.stdout.split("\n")
    tc = TrainConfig()
    for ln in [x for x in lines if x.startswith("lr ")]:
        _, step, val = ln.split()
        assert np.float32(float(val)) == np.float32(engine.learning_rate(int(step), tc))
    lcg = engine.lcg_random_vec(8, 0.5)
    for ln in [x for x in lines if x.startswith("lcg ")]:
        _, i, val = ln.split()
        assert np.float32(float(val)) == lcg[int(i)]
    tp = [tuple(int(x) for x in ln.split()[2:]) for ln in lines if ln.startswith("tp ")]
    assert tp == [engine.tp_shard(52, 17920, 8, r) for r in range(8)]
    assert ctypes.c_int  # the ctypes binding and the C program agree on every value above
