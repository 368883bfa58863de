"""The C-ABI library loads without a GPU, exports every entry point the
header declares, and its ctypes mirror matches the C struct layout."""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from barellm_b200 import _native as nat

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions() -> list[str]:
    names = []
    for h in HEADERS:
        names += re.findall(r"^BL_API\s+[\w\s\*]+?\b(bl_\w+)\s*\(", h.read_text(), flags=re.M)
    return names


def test_header_declares_the_expected_entry_points():
    assert sorted(declared_functions()) == sorted(nat.EXPORTED)


def test_library_exports_every_declared_symbol(native_lib):
    for name in declared_functions():
        assert hasattr(native_lib, name), name
    if shutil.which("nm"):
        out = subprocess.run(["nm", "-D", "--defined-only", str(nat.LIB_PATH)], capture_output=True, text=True).stdout
        exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
        assert set(declared_functions()) <= exported


def test_host_only_entry_points_work_without_gpu(native_lib):
    assert native_lib.bl_abi_version() == 1
    # split-K workspace: 64 rows, 16 q heads, D 128, up to 4096 tokens -> 8 chunks per row
    ws = native_lib.bl_paged_decode_workspace_bytes(64, 16, 128, 16, 4096)
    assert ws >= 64 * 8 * 16 * 128 * 4
    assert native_lib.bl_paged_decode_workspace_bytes(0, 16, 128, 16, 4096) == 0
    assert native_lib.bl_decode_path(nat.BL_BF16, 128, 16, 16, 8) == 1
    assert native_lib.bl_decode_path(nat.BL_BF16, 128, 16, 32, 8) == 1
    assert native_lib.bl_decode_path(nat.BL_F32, 128, 16, 16, 8) == 0
    assert native_lib.bl_decode_path(nat.BL_BF16, 64, 16, 16, 8) == 0
    assert native_lib.bl_prefill_path(nat.BL_BF16, 128, 16, 32, 8) == 1
    assert native_lib.bl_prefill_path(nat.BL_F32, 128, 16, 32, 8) == 0


def test_argument_errors_are_reported_before_any_launch(native_lib):
    a = nat.AppendArgs()  # all-zero: null pools
    rc = native_lib.bl_paged_append(ctypes.byref(a), None)
    assert rc == nat.BL_ERR_ARG
    assert "null" in nat.last_error()
    d = nat.DecodeArgs()
    assert native_lib.bl_paged_decode(ctypes.byref(d), None) == nat.BL_ERR_ARG


PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "barellm_b200.h"
#define F(s, f) printf(#s " " #f " %zu\n", offsetof(s, f));
#define S(s) printf(#s " sizeof %zu\n", sizeof(s));
int main(void) {
%s
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc unavailable")
def test_ctypes_structs_match_c_layout(tmp_path):
    lines = []
    for cname, py in nat.STRUCTS.items():
        lines.append(f"  S({cname})")
        for fname, _ in py._fields_:
            lines.append(f"  F({cname}, {fname})")
    src = tmp_path / "probe.c"
    src.write_text(PROBE.replace("%s", "\n".join(lines)))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    for line in out.splitlines():
        cname, field, value = line.split()
        py = nat.STRUCTS[cname]
        if field == "sizeof":
            assert ctypes.sizeof(py) == int(value), cname
        else:
            assert getattr(py, field).offset == int(value), (cname, field)
