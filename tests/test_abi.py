"""The C ABI library: it loads without a GPU and exports every entry point
include/wsp_decoder.h and include/wsp_encoder.h declare, with no call that
needs a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", name) for name in ("wsp_decoder.h", "wsp_encoder.h")]


def declared_functions():
    names = set()
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(header).read(), flags=re.S)
        names |= set(re.findall(r"\b(wsp_[a-z_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_the_decoder_entry_points():
    names = declared_functions()
    for required in ("wsp_decoder_create", "wsp_decoder_set_tensor", "wsp_decoder_begin_sequence",
                     "wsp_decoder_step", "wsp_decoder_transcribe", "wsp_argmax"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from whispereacp_b200._native import LIBRARY_PATH, SIGNATURES, library
    lib = library()
    assert os.path.dirname(LIBRARY_PATH) == os.path.join(ROOT, "whispereacp_b200")
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} is declared but not exported"
        assert name in SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version_and_error_text_without_a_device():
    from whispereacp_b200._native import library
    lib = library()
    assert lib.wsp_abi_version() == 1
    assert isinstance(lib.wsp_last_error(), bytes)


def test_header_declares_the_encoder_entry_points():
    names = declared_functions()
    for required in ("wsp_encoder_create", "wsp_encoder_set_tensor", "wsp_encoder_set_filters",
                     "wsp_encoder_log_mel", "wsp_encoder_encode", "wsp_encoder_encode_samples"):
        assert required in names


def test_null_arguments_are_refused_before_any_device_work():
    from whispereacp_b200._native import WSP_INVALID_ARGUMENT, library
    lib = library()
    assert lib.wsp_encoder_create(None, 0, 1, None) == WSP_INVALID_ARGUMENT
    assert lib.wsp_encoder_encode(None, None, None) == WSP_INVALID_ARGUMENT
    assert lib.wsp_decoder_create(None, 0, 1, 1, None) == WSP_INVALID_ARGUMENT
    assert b"NULL" in lib.wsp_last_error()
    assert lib.wsp_decoder_step(None, None, 1, None, None, None) == WSP_INVALID_ARGUMENT
    assert lib.wsp_decoder_begin_sequence(None, None, 0) == WSP_INVALID_ARGUMENT


def test_the_product_does_not_link_the_oracle():
    """The CUDA library and the package never reach oracle/ (it is the checker)."""
    package = os.path.join(ROOT, "whispereacp_b200")
    for folder, _, files in os.walk(package):
        for name in files:
            if name.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(folder, name)).read()
                assert "oracle" not in text.replace("oracle/", "").lower() or name == "_native.py", name
