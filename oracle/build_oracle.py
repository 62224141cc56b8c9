"""Build the oracle's C helper (oracle/dequant.c) into oracle/_build/liboracle_dequant.so with gcc.

Test infrastructure (the checker side): `__graft_entry__.build()` calls build(); the oracle also
builds it on first use when the library is missing or older than its source. Portable flags only
(no -march=native): the library is built once and also runs on other hosts.
"""
from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "dequant.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle_dequant.so")


def up_to_date() -> bool:
    return os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC)


def build(force: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the oracle helper")
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + f".tmp{os.getpid()}"
    subprocess.run([cc, "-O3", "-fPIC", "-shared", "-o", tmp, SRC, "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
