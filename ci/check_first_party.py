"""The product is this repository's own code: no Triton / TileLang kernels or torch.compile on the
package's paths, no vendored kernel libraries, and no compiled binaries (cubin, fatbin, shared
objects, object files) or profiler reports tracked by git.  Exit 1 and list what is found.

    python ci/check_first_party.py
"""
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BINARY = (".so", ".o", ".a", ".cubin", ".fatbin", ".ptx", ".ncu-rep", ".nsys-rep", ".qdrep")
FORBIDDEN_IMPORTS = re.compile(r"^\s*(import|from)\s+(triton|tilelang|flash_attn|flashinfer|fla)\b", re.M)
COMPILE = re.compile(r"torch\.compile\(")


def tracked_files():
    out = subprocess.run(["git", "ls-files"], cwd=ROOT, capture_output=True, text=True, check=True).stdout
    return [f for f in out.splitlines() if f]


def check():
    bad = []
    for f in tracked_files():
        if f.endswith(BINARY):
            bad.append(f"{f}: compiled binary or profiler report tracked")
        if f.startswith("trida_stack_b200/") and f.endswith(".py"):
            with open(os.path.join(ROOT, f), encoding="utf-8") as fh:
                src = fh.read()
            if FORBIDDEN_IMPORTS.search(src):
                bad.append(f"{f}: imports a third-party kernel library")
            if COMPILE.search(src):
                bad.append(f"{f}: uses torch.compile")
    return bad


def main():
    bad = check()
    for b in bad:
        print(b)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
