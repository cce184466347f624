"""The C-ABI library loads without a GPU and exports every symbol that
include/*.h declares; the Python binding covers the same set."""
import ctypes
import re
import subprocess

from conftest import ROOT

from cutilecpu_b200 import _lib


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^MK_API\s+[\w\s\*]+?\b(mk_\w+)\s*\(", text, flags=re.M))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("mk_vadd_f32", "mk_mapreduce_f32", "mk_sum_sq_f32", "mk_gather_f32",
                     "mk_hist_u32", "mk_last_error", "mk_error_poll"):
        assert required in names


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(declared_symbols()) if not hasattr(L, n)]
    assert not missing, f"libkernels.so lacks {missing}"


def test_binding_matches_header():
    assert set(_lib.SIGNATURES) == declared_symbols()


def test_version_and_last_error_without_gpu():
    L = _lib.lib()
    assert L.mk_version() >= 100
    assert isinstance(L.mk_last_error(), bytes)


def test_library_has_no_oracle_dependency():
    # the product library neither exports nor links the CPU oracle: read its
    # dynamic symbol table and its DT_NEEDED entries (names only)
    syms = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], check=True,
                          capture_output=True, text=True).stdout
    names = {line.split()[-1] for line in syms.splitlines() if line.strip()}
    assert not any(n.startswith(("or_", "mlirb_")) for n in names)
    dyn = subprocess.run(["readelf", "-d", str(_lib.LIB_PATH)], check=True,
                         capture_output=True, text=True).stdout
    needed = re.findall(r"\(NEEDED\).*\[(.+?)\]", dyn)
    assert needed and not any("oracle" in n for n in needed)
