"""CPU: the C ABI library loads and exports every entry point that
include/zkv.h declares; the ctypes mirrors of the ABI structs have the C
compiler's size and field offsets (no GPU work is launched)."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT
from zoomkv_revision_b200 import _lib

HEADER = os.path.join(ROOT, "include", "zkv.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(zkv_\w+)\s*\(", src, flags=re.M)))


def test_reference_select_ws_bytes():
    lib = _lib.lib()
    n = lib.zkv_reference_select_ws_bytes(64, 2040, 816, 244)
    assert n % 256 == 0 and n >= 64 * (128 * 2 + 2040 * 4 + 816 * (8 + 4 + 1 + 16 * 12) + 244 * 8)
    assert lib.zkv_reference_select_ws_bytes(-1, 1, 1, 1) == 0


def test_every_declared_symbol_is_exported_and_bound():
    names = declared()
    assert len(names) >= 20
    lib = _lib.lib()
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.exported_symbols(), n
    assert set(_lib.exported_symbols()) == set(names)
    assert lib.zkv_version() >= 100
    assert lib.zkv_status_string(6).decode()


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layouts_match_c(tmp_path):
    structs = {"zkv_page_layer": _lib.ZkvPageLayer, "zkv_rq_layout": _lib.ZkvRqLayout,
               "zkv_ref_layer": _lib.ZkvRefLayer, "zkv_peer_seg": _lib.ZkvPeerSeg,
               "zkv_raw_layer": _lib.ZkvRawLayer, "zkv_quest_large": _lib.ZkvQuestLarge,
               "zkv_raw_split": _lib.ZkvRawSplit}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for cname, cls in structs.items():
        lines.append(f'printf("%zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("%zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    c = tmp_path / "abi.c"
    c.write_text("\n".join(lines))
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-o", str(exe), str(c)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    i = 0
    for cname, cls in structs.items():
        assert vals[i] == ctypes.sizeof(cls), cname
        i += 1
        for f, _ in cls._fields_:
            assert vals[i] == getattr(cls, f).offset, (cname, f)
            i += 1


def test_status_on_bad_arguments_without_gpu():
    """Argument checks run before any launch and return ZKV_ERR_ARG."""
    lib = _lib.lib()
    assert lib.zkv_topk_f32(None, -1, 10, 10, 1, None, None) == 1
    assert lib.zkv_rq_encode(None, 128, 1, 1, 0, None, None, None) == 1
    assert lib.zkv_collision_topk(None, None, 1, 1, None, 1, 1, None, None, None) == 1
    assert lib.zkv_h2d_gather_kv(None, None, 1, 1, None, 1, 1, 0, None, None, 1, 0, None, None) == 1
    assert lib.zkv_peer_put(None, 1, None, 0, 0, 1, None, None, 0, None) == 1
    assert lib.zkv_peer_wait(None, None, 1, None, None) == 1
    assert lib.zkv_peer_handle_bytes() == 64
