"""The C-ABI library loads and exports every entry point declared in
include/helm_b200.h (no GPU needed; nothing is computed)."""
import os
import re

from helm_b200 import _capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "helm_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(helm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "helm_paged_decode_attention" in names
    assert "helm_kv_append" in names


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for name in _declared():
        assert hasattr(lib, name), name


def test_binding_covers_every_declared_symbol():
    assert sorted(_capi.exported_symbols()) == _declared()


def test_status_strings_and_version():
    lib = _capi.lib()
    assert lib.helm_version() >= 100
    assert lib.helm_status_string(0) == b"ok"
    assert lib.helm_status_string(2) == b"unsupported shape or dtype"
