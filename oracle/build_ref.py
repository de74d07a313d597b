"""Test infrastructure: build the reference engine's host sampler for parity checks.

Compiles llmy_cuda/src/llmy.cpp of a reference checkout (``LLMY_REFERENCE``;
by default the directory ``reference`` beside this repository) with g++ against its own
headers and the CUDA headers, and links ``oracle/_ref/libllmy_ref.so``.  Only
``llmy_sample`` (llmy.cpp:132-202, a pure host function) is ever called from it:
the engine entry points it also contains reference model code that is not
linked (the library is opened with lazy binding).  Nothing in the product loads
this library; tests/golden/make_llmy_sample.py uses it to produce the committed
golden vectors.  Without a reference checkout ``build_ref`` returns None.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libllmy_ref.so"


def reference_root() -> Path:
    return Path(os.environ.get("LLMY_REFERENCE",
                        Path(__file__).resolve().parents[1].parent / "reference"))


def build_ref() -> Path | None:
    """Compile the reference sampler library if the reference checkout exists."""
    ref = reference_root()
    src = ref / "llmy_cuda" / "src" / "llmy.cpp"
    if not src.exists():
        return None
    cxx = shutil.which("g++")
    if cxx is None:
        raise RuntimeError("g++ not found: cannot build the reference sampler")
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    OUT.mkdir(exist_ok=True)
    if LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    obj = OUT / "llmy.o"
    subprocess.run([cxx, "-O2", "-fPIC", "-std=c++17", f"-I{ref / 'llmy_cuda' / 'include'}",
                    f"-I{cuda / 'include'}", "-c", str(src), "-o", str(obj)], check=True)
    subprocess.run([cxx, "-shared", "-o", str(LIB), str(obj), f"-L{cuda / 'lib64'}", "-lcudart",
                    "-lcublas"], check=True)
    return LIB


if __name__ == "__main__":
    print(build_ref())
