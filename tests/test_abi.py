"""The C-ABI boundary without a GPU: the library loads, exports every
function ``include/th_b200.h`` declares, and the ctypes structs used by the
Python runtime have exactly the C layout (checked by compiling the header
with gcc and printing ``sizeof``/``offsetof``).  No compute entry point is
called here."""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess

import pytest

from conftest import REPO

HEADER = REPO / "include" / "th_b200.h"

STRUCTS = {
    "th_rowstat_args": "RowstatArgs", "th_rmsnorm_args": "RmsnormArgs", "th_gemm_args": "GemmArgs",
    "th_attention_args": "AttentionArgs", "th_conv1d_args": "Conv1dArgs", "th_ssd_args": "SsdArgs",
    "th_embedding_args": "EmbeddingArgs",
}


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\*?\s+\*?(th_[a-z0-9_]+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    fns = declared_functions()
    for f in ("th_gemm", "th_attention", "th_ssd", "th_ssd_workspace_size", "th_rmsnorm", "th_rowstat", "th_conv1d",
              "th_embedding", "th_ssd_noalloc", "th_selftest_bounded_wait", "th_version", "th_last_error_string",
              "th_device_error"):
        assert f in fns, fns


def test_library_exports_every_declared_symbol():
    from torch_helion.b200 import lib

    so = lib.load()
    missing = [f for f in declared_functions() if not hasattr(so, f)]
    assert not missing, missing
    assert set(lib.EXPORTED_SYMBOLS) == set(declared_functions())
    assert lib.version()


def test_workspace_size_is_host_only():
    from torch_helion.b200 import lib

    a = lib.ssd_workspace_size(4, 2048, 24, 64, 128, 256)
    b = lib.ssd_workspace_size(8, 2048, 24, 64, 128, 256)
    assert a > 0 and abs(b - 2 * a) <= 512


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_layout_matches_header(tmp_path):
    from torch_helion.b200 import lib

    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, pname in STRUCTS.items():
        st = getattr(lib, pname)
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in st._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    got = {}
    for line in out.splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, pname in STRUCTS.items():
        st = getattr(lib, pname)
        assert ctypes.sizeof(st) == got[(cname, "size")], cname
        for field, _ in st._fields_:
            assert getattr(st, field).offset == got[(cname, field)], (cname, field)
