"""CPU checks of the C ABI boundary: the library loads, exports every symbol the
public header declares, the ctypes table matches the header, and the
host-side validation answers without touching a GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "akv_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?(?:int|size_t|char\s*\*|const char\s*\*)\s*\*?\s*(akv_\w+)\s*\(",
                       src, flags=re.M)
    return sorted(set(names))


def test_header_parses():
    names = header_functions()
    assert "akv_quantize" in names and "akv_mixed_decode" in names
    assert len(names) >= 14


def test_library_exports_every_header_symbol():
    from akv import _C
    lib = _C.load()
    for name in header_functions():
        assert hasattr(lib, name), f"{name} missing from {_C.LIB_PATH}"


def test_ctypes_table_matches_header():
    from akv import _C
    assert sorted(_C.SIGNATURES) == header_functions()


def test_version_and_strerror():
    from akv import _C
    lib = _C.load()
    assert lib.akv_abi_version() == 3
    assert _C.strerror(0) == "ok"
    for code in range(-1, -9, -1):
        assert _C.strerror(code) != "unknown status"


def test_layout_offsets_aligned():
    from akv import _C
    for kb in (2, 3, 4):
        for vb in (2, 3, 4):
            for n in (0, 1, 3, 8):
                L = _C.warm_layout(128, kb, vb, n)
                assert L.bytes % 16 == 0
                for f in ("kc", "vc", "ks", "kz", "vs", "vz", "mask", "ko", "vo", "vd"):
                    assert getattr(L, f) % 16 == 0, f
                assert L.mask % 16 == 0 and L.flags == L.mask + 4 and L.ki == L.mask + 8
                assert L.vi == L.ki + 2 * n and L.vi + 2 * n <= L.ko
                assert L.vc == 32 * 128 * kb // 8


def test_host_validation_without_gpu():
    """Bad arguments are rejected on the host with the documented codes (nothing launched)."""
    from akv import _C
    lib = _C.load()
    assert lib.akv_warm_layout_init(128, 5, 3, 0, ctypes.byref(_C.WarmLayout())) == -2
    assert lib.akv_warm_layout_init(100, 3, 3, 0, ctypes.byref(_C.WarmLayout())) == -1
    d = _C.QDest()
    assert lib.akv_quantize(None, 0, 0, 0, None, 0, 0, 1, 1, 1, 128, 3, 1, 32, 0, ctypes.byref(d), None, None) == -7
    assert lib.akv_quantize(16, 0, 0, 0, None, 0, 0, 1, 1, 1, 128, 9, 1, 32, 0, ctypes.byref(d), None, None) == -2
    assert lib.akv_quantize(16, 0, 0, 0, None, 0, 0, 1, 1, 1, 100, 3, 1, 32, 0, ctypes.byref(d), None, None) == -1
    assert lib.akv_quantize(8, 0, 0, 0, None, 0, 0, 1, 1, 1, 128, 3, 1, 32, 0, ctypes.byref(d), None, None) == -3
    assert lib.akv_mixed_decode(16, 0, 0, None, None, 0, 0, 0, 0, None, None, 0, 0, None, 0, None,
                                1, 8, 2, 96, 1.0, 16, 0, 0, None, None, None, 0, None, None) == -4
    assert lib.akv_decode_workspace_bytes(1, 12, 2, 128, 512, 112) > 0
    assert lib.akv_decode_workspace_bytes(1, 12, 5, 128, 512, 112) == 0
    assert lib.akv_select_bottomk(None, 10, 3, 0, 0, None, None, 0, None) == -7
    assert lib.akv_cold_copy(16, 8, 16, 16, 16, 1, 0, None, None) == -1
    # an index list needs the source length it is checked against (n_src > 0)
    assert lib.akv_quantize(16, 0, 0, 0, 16, 0, 0, 1, 1, 1, 128, 3, 1, 32, 0, ctypes.byref(d), None, None) == -1
    assert lib.akv_dequantize(ctypes.byref(d), 16, 0, 0, 1, 1, 1, 128, 3, 1, 0, 16, 0, 0, 0, None, None) == -7
    assert lib.akv_gather_rows(16, 0, 0, 16, 0, 16, 1, 1, 1, 16, 16, 0, 0, 16, None, None) == -1
    assert lib.akv_abi_version() == 3


def test_layer_step_struct_matches_header(tmp_path):
    """The ctypes mirror of akv_layer_step has the header's size and field offsets."""
    import shutil
    import subprocess
    from akv import _C
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f[0] for f in _C.LayerStep._fields_]
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "akv_b200.h"\nint main(void){\n'
                   + 'printf("%zu\\n", sizeof(akv_layer_step));\n'
                   + "".join(f'printf("%zu\\n", offsetof(akv_layer_step, {f}));\n' for f in fields) + "return 0;}\n")
    exe = tmp_path / "sz"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert out[0] == ctypes.sizeof(_C.LayerStep)
    assert out[1:] == [getattr(_C.LayerStep, f).offset for f in fields]


def test_decode_args_struct_matches_header(tmp_path):
    import shutil
    import subprocess
    from akv import _C
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f[0] for f in _C.DecodeArgs._fields_]
    src = tmp_path / "da.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "akv_b200.h"\nint main(void){\n'
                   + 'printf("%zu\\n", sizeof(akv_decode_args));\n'
                   + "".join(f'printf("%zu\\n", offsetof(akv_decode_args, {f}));\n' for f in fields) + "return 0;}\n")
    exe = tmp_path / "da"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert out[0] == ctypes.sizeof(_C.DecodeArgs)
    assert out[1:] == [getattr(_C.DecodeArgs, f).offset for f in fields]
