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
    assert ctypes.sizeof(_lib.LayerStats) == 10 * 8 + 8 + 5 * 8 + 6 * 8 + 3 * 8 + 8 + 8 + 8 + 8 + 9 * 8 + 9 * 8 + 8
    # 6 int32, 2 int64, 4 int32, 14 pointers
    assert ctypes.sizeof(_lib.Planner) == 24 + 16 + 16 + 16 * 8 + 8  # + order_cap, padded


def test_plain_c_host_links_and_struct_layouts_match(tmp_path):
    """A C99 program (no C++, no torch) includes the header, links
    libferryb.so, calls it, and prints every struct's size and field offsets;
    the ctypes mirrors must agree field by field."""
    import ctypes
    import shutil
    import subprocess
    import pytest
    if shutil.which('gcc') is None:
        pytest.skip('gcc not available')
    mirrors = {'ferryb_planner': _lib.Planner, 'ferryb_layout_summary': _lib.LayoutSummary,
               'ferryb_layout_args': _lib.LayoutArgs, 'ferryb_layer_config': _lib.LayerConfig,
               'ferryb_layer_stats': _lib.LayerStats}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "ferryb.h"', 'int main(void) {',
             '  if (ferryb_version() < 1 || ferryb_last_error() == NULL) return 1;']
    for cname, py in mirrors.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ['  return 0;', '}']
    src = tmp_path / 'abi.c'
    src.write_text('\n'.join(lines) + '\n')
    exe = tmp_path / 'abi'
    libdir = str(_lib.LIB_PATH.parent)
    subprocess.run(['gcc', '-std=c99', '-Wall', '-Werror', '-pedantic', f'-I{ROOT / "include"}', str(src),
                    '-o', str(exe), f'-L{libdir}', '-lferryb', f'-Wl,-rpath,{libdir}'], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split('\n')
    got = {tuple(line.split()[:2]): int(line.split()[2]) for line in out if line}
    for cname, py in mirrors.items():
        assert got[(cname, 'size')] == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, f'{cname}.{field}'
