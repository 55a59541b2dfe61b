"""The Node-API addon that INTEGRATION.md gives a maintainer (the binding a p0pc0rn host would add) compiles against
the library's C header: its C++ blocks are extracted from INTEGRATION.md and compiled with g++ -fsyntax-only, with the
Node-API declarations it uses from tests/napi_stub (no Node toolchain exists here). A field renamed or a signature
changed in include/p0mm.h fails this test until the documented binding follows."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def addon_source():
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        text = f.read()
    section = text[text.index("## N-API addon"):text.index("## JS side")]
    blocks = re.findall(r"```cpp\n(.*?)```", section, re.S)
    assert len(blocks) >= 2, "the addon's C++ blocks"
    return "\n".join(blocks)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_addon_compiles_against_header(tmp_path):
    src = tmp_path / "p0mm_napi.cc"
    src.write_text(addon_source())
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Wno-unused-function",
                        "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "tests", "napi_stub"), str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]


def test_tuning_variables_documented():
    """Every environment variable the library reads (a tuning override or switch) has a row in INTEGRATION.md's table,
    and the table names none that the library no longer reads."""
    csrc = os.path.join(ROOT, "p0pc0rn_b200", "csrc")
    read = set()
    for f in os.listdir(csrc):
        if f.endswith((".cu", ".cuh", ".h", ".cc")):
            read |= set(re.findall(r'getenv\("(P0MM_\w+)"\)', open(os.path.join(csrc, f)).read()))
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        documented = set(re.findall(r"^\| `(P0MM_\w+)", f.read(), re.M))
    assert read, "the library reads tuning variables"
    assert read == documented, (sorted(read - documented), sorted(documented - read))
