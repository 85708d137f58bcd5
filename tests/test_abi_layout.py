"""The ctypes mirrors in nurostream_b200/_lib.py lay their structs out exactly as a C compiler does
from include/ns_b200.h: every field's offset and every struct's size, checked against gcc."""
import ctypes as C
import shutil
import subprocess

import pytest

from nurostream_b200 import _lib

STRUCTS = {
    "ns_moe_layer_t": _lib.MoeLayerParams,
    "ns_dense_seg_t": _lib.DenseSeg,
    "ns_dense_gemv_t": _lib.DenseGemvParams,
    "ns_attn_decode_t": _lib.AttnDecodeParams,
    "ns_l2_prefetch_t": _lib.L2Prefetch,
    "ns_attn_block_t": _lib.AttnBlockParams,
    "ns_peer_reduce_t": _lib.PeerReduceParams,
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layouts_match_the_header(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{_lib.HEADER}"', "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for line in out:
        if line:
            *key, val = line.split()
            got[tuple(key)] = int(val)
    for cname, cls in STRUCTS.items():
        assert got[(cname, "size")] == C.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, f"{cname}.{fname}"
