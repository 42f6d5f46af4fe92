"""The C-ABI library loads without a GPU and exports every symbol that
include/ferryb.h declares; the Python binding covers each of them."""
import re
from pathlib import Path

from ferry_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / 'include' / 'ferryb.h').read_text()
    return sorted(set(re.findall(r'FERRYB_API\s+[\w\s\*]+?\b(ferryb_\w+)\s*\(', text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert 'ferryb_plan_layer' in names and 'ferryb_execute_experts' in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f'not exported: {missing}'


def test_binding_signatures_cover_header():
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_version_and_error_text():
    lib = _lib.lib()
    assert lib.ferryb_version() >= 1
    assert isinstance(lib.ferryb_last_error(), bytes)


def test_struct_sizes_match_c_layout():
    import ctypes
    # 8 int32 + 2 x 256 int32 + 3 x 32 int32
    assert ctypes.sizeof(_lib.LayoutSummary) == 4 * (8 + 512 + 96)
    assert ctypes.sizeof(_lib.LayerConfig) == 14 * 4
    assert ctypes.sizeof(_lib.LayerStats) == 10 * 8 + 8 + 5 * 8 + 6 * 8 + 3 * 8 + 8 + 8 + 8 + 8 + 9 * 8 + 9 * 8
    # 6 int32, 2 int64, 4 int32, 14 pointers
    assert ctypes.sizeof(_lib.Planner) == 24 + 16 + 16 + 16 * 8 + 8  # + order_cap, padded
