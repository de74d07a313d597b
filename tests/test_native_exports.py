"""CPU: the C-ABI library loads and exports every symbol include/*.h declares."""
import ctypes
import re
from pathlib import Path

from hybrid_llm_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^\s*(?:int32_t|int64_t|void)\s+(llmyb_\w+)\s*\(", text, re.M))
    return names


def test_header_declares_entry_points():
    assert "llmyb_route" in declared_symbols()


def test_library_exports_every_declared_symbol():
    handle = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [n for n in sorted(declared_symbols()) if not hasattr(handle, n)]
    assert not missing, f"symbols declared in include/ but not exported: {missing}"


def test_binding_table_matches_header():
    assert set(_native.SIGNATURES) == declared_symbols()
    _native.lib()  # binds argtypes for every entry
