"""TEST INFRASTRUCTURE — struct layouts (sizeof / offsetof of every field) of the moert island ABI.

`python tests/golden/abi_layout.py --reference <moert include dir>` measures the layouts the
reference header declares (moert/include/moert/cuda.h) and writes moert_abi_layout.json next to
this file; tests/test_abi.py measures the same fields through this repository's
include/moert_cuda.h and compares. Field names come from this repository's header; a field the
reference lacks fails the reference compile.
"""
from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OURS = os.path.join(ROOT, "include", "moert_cuda.h")
STRUCTS = ["moert_cuda_config", "moert_coldcpu_call", "moert_coldffn_job", "moert_mm_call", "moert_ffn_moe_host",
           "moert_ffn_moe_args", "moert_cuda_stats", "moert_cuda_dir_stats"]


def fields(header: str, name: str) -> list[str]:
    src = re.sub(r"/\*.*?\*/", "", open(header).read(), flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    m = re.search(r"typedef\s+struct\s+" + name + r"\s*\{(.*?)\}\s*" + name + r"\s*;", src, flags=re.S)
    if not m:
        raise ValueError(f"struct {name} not found in {header}")
    out = []
    for stmt in m.group(1).split(";"):
        stmt = stmt.strip()
        if not stmt:
            continue
        fp = re.search(r"\(\s*\*\s*(\w+)\s*\)", stmt)
        if fp:
            out.append(fp.group(1))
            continue
        for decl in stmt.split(","):
            ident = re.findall(r"(\w+)\s*(?:\[[^\]]*\])?\s*$", decl.strip())
            if ident:
                out.append(ident[0])
    return out


def measure(include_line: str, include_dirs: list[str]) -> dict:
    prog = ["#include <stdio.h>", "#include <stddef.h>", "#include <stdint.h>", include_line, "int main(void) {"]
    for s in STRUCTS:
        prog.append(f'    printf("{s} sizeof %zu\\n", sizeof({s}));')
        for f in fields(OURS, s):
            prog.append(f'    printf("{s} {f} %zu\\n", offsetof({s}, {f}));')
    prog += ["    return 0;", "}"]
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        open(c, "w").write("\n".join(prog) + "\n")
        subprocess.run(["gcc", "-std=c11", *[f"-I{i}" for i in include_dirs], c, "-o", exe], check=True)
        lines = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    out: dict = {}
    for ln in lines:
        if ln:
            s, f, v = ln.split()
            out.setdefault(s, {})[f] = int(v)
    return out


def ours() -> dict:
    return measure('#include "moert_cuda.h"', [os.path.dirname(OURS)])


if __name__ == "__main__":
    if len(sys.argv) != 3 or sys.argv[1] != "--reference":
        sys.exit("usage: abi_layout.py --reference <dir containing moert/cuda.h>")
    ref = measure('#include "moert/cuda.h"', [sys.argv[2]])
    with open(os.path.join(HERE, "moert_abi_layout.json"), "w") as fh:
        json.dump(ref, fh, indent=1, sort_keys=True)
    print(f"wrote {sum(len(v) for v in ref.values())} entries")
