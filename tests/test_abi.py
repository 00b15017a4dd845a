"""The C-ABI library builds, loads and exports every symbol ``include/dels_b200.h``
declares; argument errors are reported without touching a GPU.  CPU only."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "dels_b200.h"


def _declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"DELS_API\s+[\w\s\*]+?\b(dels_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from dels_b200 import _lib, build

    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = _declared()
    assert len(names) >= 19
    for must in ("dels_draft_score_bf16", "dels_fused_argmax_bf16", "dels_accept_offsets", "dels_keys_decode",
                 "dels_draft_score_f32", "dels_rnn_rank_states_bf16", "dels_fused_argmax_base_bf16"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    from dels_b200 import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (dels_\w+)", out))
    declared = set(_declared())
    assert declared <= exported, declared - exported
    assert exported <= declared, exported - declared  # nothing undocumented
    assert set(_lib.SIGNATURES) == declared  # the Python binding covers the whole ABI
    for name in declared:
        assert getattr(lib, name) is not None


def test_pure_host_entry_points(lib):
    from dels_b200 import _lib

    assert lib.dels_version() == 1
    assert lib.dels_status_string(_lib.DELS_ERR_ALIGNMENT) == b"misaligned pointer or leading dimension"
    assert _lib.query("dels_score_workspace_bytes", 512, 4096, 256) > 512 * 256 * 2
    assert _lib.query("dels_rank_workspace_bytes", 0, 1, 1) == _lib.DELS_WS_HEADER_BYTES
    assert _lib.query("dels_rnn_workspace_bytes", 512, 16, 4096, 256) >= 8192 * 256 * 4
    # vocabulary-sized F.linear: the GEMM writes bf16 itself, no split-K partials
    assert _lib.query("dels_linear_workspace_bytes", 14, 4096, 151936) == _lib.DELS_WS_HEADER_BYTES
    # the correction layer always finalises from partials, even when K is a single block
    assert _lib.query("dels_correction_mid_tc_workspace_bytes", 40, 64, 48) >= \
        _lib.DELS_WS_HEADER_BYTES + 40 * 48 * 4


def test_plain_c_host_links_and_calls(lib, tmp_path):
    """The header is C99 and a C program links against the library directly (no Python,
    no torch): the boundary a cgo / JNI / N-API binding would wrap."""
    import shutil

    from dels_b200 import _lib

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(
        "#include <stdio.h>\n#include \"dels_b200.h\"\n"
        "int main(void) {\n"
        "  if (dels_version() != 1) return 2;\n"
        "  if (dels_linear_workspace_bytes(14, 4096, 151936) != DELS_WS_HEADER_BYTES) return 3;\n"
        "  if (dels_rank_workspace_bytes(0, 1, 1) != DELS_WS_HEADER_BYTES) return 4;\n"
        "  puts(dels_status_string(DELS_ERR_WORKSPACE));\n"
        "  return 0;\n}\n")
    libdir = _lib.LIB_PATH.parent
    exe = tmp_path / "host"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", str(HEADER.parent), str(src), "-L", str(libdir),
                    "-ldels_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    assert out.strip() == "workspace missing or too small"


def test_argument_errors_are_reported_before_device_work(lib):
    from dels_b200 import _lib

    # NULL keys -> invalid argument, with a message
    with pytest.raises(_lib.DelsArgumentError) as ei:
        _lib.call("dels_fused_argmax_bf16", None, 0, None, 0, None, 0, None, 0, None, None, 1, None, 4, None, 64, 64,
                  100, 0, 0, None, None, None, None, 0, None)
    assert ei.value.status in (_lib.DELS_ERR_INVALID_ARG, _lib.DELS_ERR_ALIGNMENT)
    assert lib.dels_last_error()
    # misaligned operand
    buf = (ctypes.c_char * 64)()
    addr = ctypes.addressof(buf) | 2
    with pytest.raises(_lib.DelsArgumentError) as ei:
        _lib.call("dels_rank_project_bf16", ctypes.c_void_p(addr), 64, ctypes.c_void_p(addr), 64, 4, 64, 8, 0, None,
                  1, None, None, ctypes.c_void_p(addr), None, None, 0, None)
    assert ei.value.status == _lib.DELS_ERR_ALIGNMENT
    # unknown activation
    with pytest.raises(_lib.DelsArgumentError):
        _lib.call("dels_rank_project_bf16", None, 0, None, 0, 4, 64, 8, 7, None, 1, None, None, None, None, None, 0,
                  None)
    # commit_extra outside {0, 1}
    with pytest.raises(_lib.DelsArgumentError):
        _lib.call("dels_accept_offsets", None, 0, None, 0, 1, 1, 2, None, None, None)
    # the fused GRU-gate entry points check their operands before any device work
    with pytest.raises(_lib.DelsArgumentError) as ei:
        _lib.call("dels_gru_rank_gemv_bf16", None, 1, 0, None, 3072, None, 3072, None, None, 1, 1024, 100, None, 1024,
                  None, 256, 0, None, None, None, None, None)
    assert ei.value.status == _lib.DELS_ERR_INVALID_ARG
    with pytest.raises(_lib.DelsArgumentError) as ei:
        _lib.call("dels_gru_correction_mid_bf16", ctypes.c_void_p(addr), 1, 0, ctypes.c_void_p(addr), 3072,
                  ctypes.c_void_p(addr), 3072, None, ctypes.c_void_p(addr), 1, 1024, 100, None, 1024,
                  ctypes.c_void_p(addr), 1024, 1024, None, None, None, None, None)
    assert ei.value.status == _lib.DELS_ERR_ALIGNMENT
    # the scorer with the next GRU projection takes at most 8 rows
    ok = (ctypes.c_char * 256)()
    p = ctypes.c_void_p((ctypes.addressof(ok) + 15) & ~15)
    with pytest.raises(_lib.DelsError) as ei:
        _lib.call("dels_fused_argmax_base_gru_bf16", p, 1000, p, 64, p, 64, None, None, 1, 9, 64, 1000, 0, None,
                  None, p, 256, p, None, p, 1024, p, None)
    assert ei.value.status == _lib.DELS_ERR_UNSUPPORTED
    # the tensor-core GRU step: NULL operands, then a misaligned h_in, before any device work
    with pytest.raises(_lib.DelsArgumentError) as ei:
        _lib.call("dels_gru_step_tc_bf16", None, 1, 0, None, 3072, None, None, None, None, 16, 1024, 100, None, 0,
                  None)
    assert ei.value.status == _lib.DELS_ERR_INVALID_ARG
    with pytest.raises(_lib.DelsArgumentError) as ei:
        _lib.call("dels_gru_step_tc_bf16", p, 1, 0, p, 3072, p, None, ctypes.c_void_p(addr), p, 16, 1024, 100, None,
                  0, None)
    assert ei.value.status == _lib.DELS_ERR_ALIGNMENT
    assert _lib.query("dels_gru_step_tc_workspace_bytes", 16, 1024) > _lib.DELS_WS_HEADER_BYTES
    # fp32 scorer needs H % 4 == 0
    with pytest.raises(_lib.DelsError):
        _lib.call("dels_draft_score_f32", None, 0, None, 0, None, 0, None, 0, None, None, None, 1, None, 1, 6, 4, 10,
                  0, None, None, None, None, 0, None)


def test_no_fallback_when_library_missing(monkeypatch, tmp_path):
    from dels_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(RuntimeError, match="no non-CUDA fallback"):
        _lib.load()
