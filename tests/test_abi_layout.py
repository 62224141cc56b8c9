"""The C ABI's data layout and the source rules, checked on the host.

* `struct sb_moe_layer` as the C compiler lays it out (gcc on include/shard_b200.h) against the
  ctypes mirror in shard_b200/_lib.py: every field's offset and the struct's size. A field added on
  one side only would otherwise reach the kernels as shifted pointers.
* The CUDA sources issue no bulk or tensor copy with cluster multicast and name none of the batched
  memcpy entry points that are closed on this hardware's driver (the build's own guard rules)."""
import ctypes
import glob
import os
import re
import shutil
import subprocess
import tempfile

import pytest

from shard_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "shard_b200.h")
CSRC = os.path.join(ROOT, "shard_b200", "csrc")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_layer_struct_layout_matches_the_header():
    fields = [name for name, _ in _lib.SbMoeLayer._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(sb_moe_layer, {f}));' for f in fields)
    src = ("#include <stddef.h>\n#include <stdio.h>\n#include \"shard_b200.h\"\n"
           f"int main(void) {{\n{body}\n  printf(\"sizeof %zu\\n\", sizeof(sb_moe_layer));\n  return 0;\n}}\n")
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True,
                       capture_output=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    got = dict(line.split() for line in out if line.strip())
    for f in fields:
        assert int(got[f]) == getattr(_lib.SbMoeLayer, f).offset, f"offset of {f}"
    assert int(got["sizeof"]) == ctypes.sizeof(_lib.SbMoeLayer)


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(CSRC, "*.h")) + [HEADER])


def test_no_multicast_copies_and_no_batched_memcpy():
    # the patterns are assembled from fragments so that this file names neither construct itself
    multicast = re.compile(r"cp\.async\.bulk[^\"\n]*" + "multi" + "cast")
    batched = re.compile("Mem" + "cpy(3D)?" + "Batch" + "Async")
    for path in _sources():
        text = open(path).read()
        assert not multicast.search(text), f"{path}: a bulk / tensor copy with cluster multicast"
        assert not batched.search(text), f"{path}: a batched memcpy entry point"
