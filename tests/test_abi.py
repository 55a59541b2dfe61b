"""The C-ABI boundary on CPU (no kernel runs): libp0mm.so loads, exports every entry point include/p0mm.h declares,
and the ctypes mirror of each argument struct has the C layout (sizes and field offsets from a C program compiled
against the header with the host compiler)."""
import ctypes
import os
import re
import subprocess

import pytest

from p0pc0rn_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "p0mm.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:p0_status|const char \*)\s*(p0_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_the_known_surface():
    assert declared_functions() == sorted(L.EXPORTS)


def test_library_exports_every_declared_function():
    lib = ctypes.CDLL(L.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_string():
    v = L.load().p0_version()
    assert b"sm_100a" in v and b"gemv" in v and b"gemm" in v


STRUCTS = {
    "p0_wview": L.p0_wview,
    "p0_gemv_args": L.p0_gemv_args,
    "p0_gemvM_args": L.p0_gemvM_args,
    "p0_gemm_args": L.p0_gemm_args,
    "p0_embed_args": L.p0_embed_args,
    "p0_normadd_args": L.p0_normadd_args,
    "p0_dhead_args": L.p0_dhead_args,
    "p0_qkrope_args": L.p0_qkrope_args,
    "p0_attn_dec_args": L.p0_attn_dec_args,
}


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    d = tmp_path_factory.mktemp("abi")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "p0mm.h"', "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append('  printf("%s size %%zu\\n", sizeof(%s));' % (cname, cname))
        for f, _ in cls._fields_:
            lines.append('  printf("%s.%s %%zu\\n", offsetof(%s, %s));' % (cname, f, cname, f))
    lines += ["  return 0;", "}"]
    c = d / "layout.c"
    c.write_text("\n".join(lines) + "\n")
    exe = d / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(HEADER), str(c), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return dict(line.rsplit(" ", 1) for line in out.strip().splitlines())


@pytest.mark.parametrize("cname", sorted(STRUCTS))
def test_struct_layout_matches_header(c_layout, cname):
    cls = STRUCTS[cname]
    assert int(c_layout["%s size" % cname]) == ctypes.sizeof(cls)
    for f, _ in cls._fields_:
        assert int(c_layout["%s.%s" % (cname, f)]) == getattr(cls, f).offset, f


def test_init_without_a_device_reports_a_status():
    # on a host without a CUDA device the library returns P0_EDEVICE instead of crashing
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    lib = L.load()
    ctx = ctypes.c_void_p()
    assert lib.p0_init(0, ctypes.byref(ctx)) == L.P0_EDEVICE
    assert not ctx.value
