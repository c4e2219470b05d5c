"""The C ABI without a GPU: libtbcuda.so loads, exports every function include/tbcuda.h
declares, and the ctypes mirrors of its structs have the C layout (checked against a
probe compiled with gcc from the header itself)."""

import ctypes
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "tbcuda.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(tb_[a-z0-9_]+)\s*\(", text))


def test_library_loads_and_exports_every_declared_symbol():
    from tinybark_b200 import _lib

    names = declared()
    assert len(names) >= 15
    missing = [n for n in sorted(names) if not hasattr(_lib.lib, n)]
    assert not missing, missing
    assert set(_lib.EXPORTS) == names
    assert _lib.lib.tb_version() == 1


def test_workspace_queries_need_no_gpu():
    from tinybark_b200 import _lib

    lib = _lib.lib
    assert lib.tb_encoder_workspace_bytes(_lib.BF16, 250, 125) > 125 * 1024 * 2 * 10
    assert lib.tb_encoder_workspace_bytes(_lib.F32, 250, 125) > lib.tb_encoder_workspace_bytes(_lib.BF16, 250, 125)
    one = lib.tb_decode_workspace_bytes(_lib.BF16, 64, 1)
    assert one > 64 * 640 * 4
    assert lib.tb_decode_workspace_bytes(_lib.BF16, 64, 4) >= one
    assert lib.tb_frontend_workspace_bytes(4, 1000) >= 4 * 128 * 16
    assert _lib.tile_rows(_lib.F32)[0] == 8


def test_bad_arguments_are_rejected_without_touching_the_device():
    from tinybark_b200 import _lib

    ep = _lib.Epilogue(kind=_lib.EPI_STORE)
    assert _lib.lib.tb_gemm(7, 1, 64, 1, 4, 128, 64, ctypes.byref(ep), None, None) == 1
    assert _lib.lib.tb_gemm(_lib.BF16, None, 64, None, 4, 128, 64, ctypes.byref(ep), None, None) == 1
    assert _lib.lib.tb_gemm(_lib.F32, 8, 64, 8, 4, 100, 64, ctypes.byref(ep), None, None) == 3
    # text: negative lanes, a missing piece table
    assert _lib.lib.tb_text_offsets(None, 8, None, -1, None, 10, 8, None, None) == 1
    assert _lib.lib.tb_text_offsets(8, 8, 8, 4, None, 10, 8, None, None) == 1
    assert _lib.lib.tb_text_bytes(8, 8, 8, 4, 8, None, 5, 10, 8, 8, 100, None) == 1
    # block-scaled: K not a multiple of 512, N not a multiple of 128, a bad source dtype
    assert _lib.lib.tb_gemm_mx(16, 16, 16, 16, 4, 128, 1000, ctypes.byref(ep), None, None) == 1
    assert _lib.lib.tb_gemm_mx(16, 16, 16, 16, 4, 100, 1024, ctypes.byref(ep), None, None) == 1
    assert _lib.lib.tb_mx_quantize(5, 16, 1024, 4, 1024, 16, 16, None) == 1
    assert _lib.lib.tb_mx_scale_bytes(200, 1024) == 256 * 32
    assert _lib.lib.tb_encoder_workspace_bytes_mx(100, 50) > _lib.lib.tb_encoder_workspace_bytes(_lib.BF16, 100, 50)
    with pytest.raises(RuntimeError, match="bad argument"):
        _lib.check(1, "tb_gemm")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layouts_match_the_header(tmp_path):
    from tinybark_b200 import _lib

    structs = {"tb_epilogue": _lib.Epilogue, "tb_layer": _lib.Layer, "tb_model": _lib.Model, "tb_batch": _lib.Batch,
               "tb_repack_job": _lib.RepackJob, "tb_mx_weight": _lib.MXWeight}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("return 0; }")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    for line in filter(None, out):
        cname, field, value = line.split()
        cls = structs[cname]
        got = ctypes.sizeof(cls) if field == "size" else getattr(cls, field).offset
        assert got == int(value), (cname, field, got, value)
