"""CPU-side checks of the C ABI: the shared library loads and exports every symbol that
include/dollama_b200.h declares (no compute calls; no GPU needed)."""
from dollama_b200 import _lib as L


def test_library_loads():
    lib = L.lib()
    assert lib.dlm_version().decode().startswith("dollama_b200")


def test_exports_every_header_symbol():
    lib = L.lib()
    names = L.header_symbols()
    assert len(names) >= 5
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    assert set(L.header_symbols()) == set(L._SIGS), (
        set(L.header_symbols()) ^ set(L._SIGS))


def test_last_error_empty_on_fresh_thread():
    assert isinstance(L.last_error(), str)
