"""The C-ABI library loads without a GPU, exports every entry point its headers
declare, and turns bad input into statuses (no compute calls here)."""

import ctypes
import os
import re
import struct

import numpy as np
import pytest

from tests.conftest import ROOT


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nb_[a-z_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(native_built):
    lib = ctypes.CDLL(native_built)
    names = _declared("needle_b200.h") + _declared("needle_b200_debug.h")
    assert "nb_model_open" in names and "nb_batch_step" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def _open_status(path):
    import rustyneedle_b200 as nb
    from rustyneedle_b200._native import lib, nb_options

    h = ctypes.c_void_p()
    status = lib().nb_model_open(path.encode(), ctypes.byref(nb_options(-1, 0, 0, 0)), ctypes.byref(h))
    return status, lib().nb_last_error().decode()


def test_missing_file_is_an_io_error(native_built, tmp_path):
    status, message = _open_status(str(tmp_path / "absent.cact"))
    assert status == -1 and "absent.cact" in message


def test_wrong_tag_is_an_archive_error(native_built, tmp_path):
    p = tmp_path / "bad.cact"
    p.write_bytes(struct.pack("<I", 0x12345678) + b"\0" * 400)
    status, message = _open_status(str(p))
    assert status == -2 and "format tag 0x12345678" in message


def test_truncated_archives_are_archive_errors(native_built, archive_path, tmp_path):
    data = open(archive_path, "rb").read()
    for cut in (10, 200, 300, len(data) // 2):
        p = tmp_path / f"cut{cut}.cact"
        p.write_bytes(data[:cut])
        status, _ = _open_status(str(p))
        assert status == -2, cut


def test_unknown_element_kind_is_an_archive_error(native_built, archive_path, tmp_path):
    data = bytearray(open(archive_path, "rb").read())
    directory = 196 + 28 * 4
    data[directory] = 9
    p = tmp_path / "kind.cact"
    p.write_bytes(bytes(data))
    status, message = _open_status(str(p))
    assert status == -2 and "kind 9" in message


def test_a_valid_archive_needs_a_device(native_built, archive_path):
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    status, message = _open_status(archive_path)
    assert status == -10, message


def test_null_arguments_are_refused(native_built):
    from rustyneedle_b200._native import lib

    L = lib()
    assert L.nb_model_open(None, None, None) == -4
    assert L.nb_session_push(None, 1) == -4
    assert L.nb_batch_step(None, None, None, None) == -4
    assert L.nb_session_len(None) == 0


def test_product_path_has_no_cpu_fallback(tmp_path, monkeypatch):
    from rustyneedle_b200 import _native

    monkeypatch.setattr(_native, "_LIBRARY", str(tmp_path / "missing.so"))
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(ImportError):
        _native.lib()
