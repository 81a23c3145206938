"""The drop-in boundary: libqtts.so loads and exports every entry point that
include/qtts.h declares, the Python mirror declares the same set, and the
library reports errors through return codes and qtts_last_error (no GPU
compute here)."""
import ctypes
import os
import re

import pytest

import qtts

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qtts.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(qtts_[a-z0-9_]+)\s*\(", text))


def test_header_declares_the_stack_api():
    names = declared()
    for n in ("qtts_stack_create", "qtts_heads_add", "qtts_heads_digest", "qtts_lm_create", "qtts_lm_forward",
              "qtts_lm_reset", "qtts_lm_length", "qtts_talker_start", "qtts_talker_next_frame", "qtts_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(qtts.LIB_PATH)
    missing = [n for n in sorted(declared()) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_mirror_covers_the_header():
    assert declared() - {"qtts_last_error"} == set(qtts.EXPORTS)


def test_errors_are_codes_not_crashes():
    lib = qtts.lib()
    # NULL out-pointer: rejected before any CUDA call
    assert lib.qtts_device_open(0, None) == qtts.E_ARG
    assert b"NULL" in lib.qtts_last_error()
    # NULL handles are rejected, destroy(NULL) is a no-op
    assert lib.qtts_lm_forward(None, None, 1, 0, None, None) == qtts.E_ARG
    assert lib.qtts_lm_destroy(None) == 0
    assert lib.qtts_talker_next_frame(None, None, None) == qtts.E_ARG
    with pytest.raises(qtts.EQwenLm) as e:
        qtts.check(lib.qtts_heads_count(None, None))
    assert e.value.code == qtts.E_ARG


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(qtts.EQwenLm):
        qtts.load_library(str(tmp_path / "libqtts.so"))
