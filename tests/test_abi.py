"""The C-ABI library loads and exports every symbol the headers in include/ declare."""
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
HEADERS = sorted(os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h"))


def declared_symbols():
    text = "\n".join(open(h).read() for h in HEADERS)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dn_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "dn_model_forward" in syms and "dn_weights_open" in syms
    assert len(syms) >= 10


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol(pkg):
    assert set(declared_symbols()) <= set(pkg.SIGNATURES), set(declared_symbols()) - set(pkg.SIGNATURES)


def test_abi_version_and_error_string(pkg):
    lib = pkg.lib()
    assert lib.dn_abi_version() >= 100
    assert isinstance(lib.dn_last_error(), bytes)
