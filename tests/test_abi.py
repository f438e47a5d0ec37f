"""CPU: the C-ABI library builds for sm_100a, loads, and exports every entry point include/sa3b200.h declares."""
import ctypes
import os
import re

from sa3_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sa3b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bint\s+(sa3_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "sa3_gemm" in syms and "sa3_attention" in syms
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_library_exports_every_declared_symbol():
    path = build.build()
    lib = ctypes.CDLL(path)
    for s in declared_symbols():
        assert hasattr(lib, s), s


def test_version_callable_without_gpu():
    assert _lib.load().sa3_version() >= 100


def test_host_side_argument_errors_need_no_gpu():
    lib = _lib.load()
    # null pointers and bad sizes are rejected on the host before any CUDA call
    assert lib.sa3_gemm(None, None, None, 0, 0, 0, 0, 0, 0, 0, None, None, None, None) == -1
    assert lib.sa3_attention(None, None, None, None, None, None, None, None, None, 1, 1, 1, 1, 1, 1, 64, 64, 64, 64,
                             64, -1, -1, 0.125, 0, None, None) == -1
    assert lib.sa3_diff_attn_swa(None, None, None, None, 0, 1, 1, 1, 64, 17, None) == -1
    assert lib.sa3_rmsnorm_modulate(None, 0, None, 0, 0, 0, 0, None, 1e-5, None, 0, 0, 0, 0, None, 0, 0, None,
                                    None, None, None, None) == -1
    assert lib.sa3_convert(None, 0, None, 0, 0, 0, 0, 0, None, None) == -1


def test_epilogue_struct_layout_matches_header(tmp_path):
    """The ctypes mirror of sa3_epilogue has the C compiler's size and field offsets."""
    import shutil
    import subprocess

    import pytest

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f for f, _ in _lib.Epilogue._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "sa3b200.h"\nint main(void) {\n'
                   '  printf("%zu\\n", sizeof(sa3_epilogue));\n'
                   + "".join(f'  printf("%zu\\n", offsetof(sa3_epilogue, {f}));\n' for f in fields)
                   + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(_lib.Epilogue)
    for f, off in zip(fields, out[1:]):
        assert getattr(_lib.Epilogue, f).offset == off, f


def test_qk_gamma_table_arguments_checked_on_host():
    """The qk-norm epilogue's gamma-table mode: bad table arguments are rejected before any CUDA call (the
    pointers below are aligned placeholders that are never dereferenced)."""
    lib = _lib.load()
    A = B = C = 0x100000

    def gemm(**kw):
        e = _lib.Epilogue()
        e.kind = _lib.EPI_QK_NORM
        e.qk_group_width = 128
        for k, v in kw.items():
            setattr(e, k, v)
        return lib.sa3_gemm(A, B, C, 256, 1536, 256, 256, 256, 1536, _lib.DT_BF16, None, None, ctypes.byref(e), None)

    assert gemm() == -1  # 12 groups of 128 columns without a table: more than 8
    assert gemm(qk_gamma_table=0x200000, qk_table_groups=0) == -1
    assert gemm(qk_gamma_table=0x200000, qk_table_groups=9, qk_rope_mask=1) == -1  # no rotary embedding in table mode
    assert gemm(qk_gamma_table=0x200004, qk_table_groups=9) == -2  # 16-byte alignment
    assert gemm(qk_group_width=96, qk_gamma_table=0x200000, qk_table_groups=9) == -1  # group width % 64
