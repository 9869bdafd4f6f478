"""C-ABI boundary checks that need no GPU: symbols, struct layout, refusals."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from cxlsparse_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "cxlsparse.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(cxs_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared()
    assert set(names) == set(_lib.exported_symbols())
    for name in names:
        assert hasattr(lib, name), name
    assert lib.cxs_abi_version() == _lib.ABI_VERSION == 4


def _c_layout(struct, fields):
    body = "\n".join(f'printf("%zu\\n", offsetof({struct}, {f}));' for f in fields)
    return body + f'\nprintf("%zu\\n", sizeof({struct}));'


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc required")
def test_ctypes_structs_match_c_layout(tmp_path):
    pairs = [("cxs_plan_geometry", _lib.PlanGeometry), ("cxs_plan_buffers", _lib.PlanBuffers),
             ("cxs_attend_geometry", _lib.AttendGeometry),
             ("cxs_attend_buffers", _lib.AttendBuffers),
             ("cxs_select_geometry", _lib.SelectGeometry)]
    source = ["#include <stdio.h>", "#include <stddef.h>", '#include "cxlsparse.h"',
              "int main(void) {"]
    for name, cls in pairs:
        source.append(_c_layout(name, [f for f, _ in cls._fields_]))
    source.append("return 0; }")
    c_file = tmp_path / "layout.c"
    c_file.write_text("\n".join(source))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(c_file), "-o", str(exe)], check=True)
    values = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                             check=True).stdout.split()]
    expected = []
    for _, cls in pairs:
        expected += [getattr(cls, f).offset for f, _ in cls._fields_] + [ctypes.sizeof(cls)]
    assert values == expected


def _geometry(**kw):
    base = dict(queries=13, heads=2, width=4, block_size=16, map_blocks=64, per_head=52,
                sort_extent=832, hot=32, max_history=131, regions=1, page_size=64,
                consumer_ctas=26, read_order=1, private_plan=0, pool_tokens=1000)
    base.update(kw)
    return _lib.PlanGeometry(**base)


def test_plan_geometry_refusals_before_any_launch():
    lib = _lib.lib()
    assert lib.cxs_plan_check(_geometry()) == _lib.OK
    assert lib.cxs_plan_check(_geometry(block_size=24)) == _lib.ERR_INVALID
    assert lib.cxs_plan_check(_geometry(per_head=65)) == _lib.ERR_INVALID
    assert lib.cxs_plan_check(_geometry(read_order=7)) == _lib.ERR_INVALID
    assert lib.cxs_plan_check(_geometry(hot=8192, sort_extent=8192)) == _lib.ERR_CAPACITY
    assert lib.cxs_plan_check(_geometry(map_blocks=1 << 19, per_head=52)) == _lib.ERR_CAPACITY
    assert lib.cxs_plan_check(_geometry(private_plan=1, width=40, per_head=520)) == \
        _lib.ERR_CAPACITY
    with pytest.raises(_lib.CapacityError):
        _lib.check(lib.cxs_plan_check(_geometry(hot=8192, sort_extent=8192)))
    with pytest.raises(ValueError):
        _lib.check(lib.cxs_plan_check(_geometry(block_size=24)))


def test_invalid_attend_arguments_are_rejected_without_a_device():
    lib = _lib.lib()
    g = _lib.AttendGeometry(queries=1, heads=2, width=4, block_size=24, physical=8)
    b = _lib.AttendBuffers()
    assert lib.cxs_fetch_attend(g, b, None) == _lib.ERR_INVALID
    g.block_size, g.gate = 16, 1
    assert lib.cxs_fetch_attend(g, b, None) == _lib.ERR_INVALID
    assert b"gate" in lib.cxs_last_error()
    g = _lib.AttendGeometry(queries=1, heads=2, width=4, block_size=16, physical=8, ctas=-1)
    assert lib.cxs_fetch_attend(g, b, None) == _lib.ERR_INVALID
    assert b"ctas" in lib.cxs_last_error()


def test_segment_select_and_exchange_arguments_are_rejected_without_a_device():
    """Candidate segments, the NSA selection geometry, window compression and
    the KV-head exchange refuse bad geometry before touching the device."""
    import ctypes

    lib = _lib.lib()
    # Segments must be whole blocks.
    g = _lib.AttendGeometry(queries=4, heads=2, width=4, block_size=64, physical=8,
                            segment_start=100, segment_tokens=128)
    assert lib.cxs_fetch_attend(g, _lib.AttendBuffers(), None) == _lib.ERR_INVALID
    assert b"segment" in lib.cxs_last_error()
    # The output layout must hold this call's heads.
    g = _lib.AttendGeometry(queries=4, heads=2, width=4, block_size=64, physical=8,
                            out_heads=2, out_head0=1)
    assert lib.cxs_fetch_attend(g, _lib.AttendBuffers(), None) == _lib.ERR_INVALID
    # NSA geometry: the window must be a multiple of the stride, the stride
    # must divide the block, forced is 0 or 1.
    q = ctypes.c_void_p(16)
    for bad in (dict(window=24, stride=16), dict(window=32, stride=24),
                dict(window=32, stride=16, forced=2)):
        sg = _lib.SelectGeometry(queries=1, heads=2, block_size=64, count=16, summaries=0,
                                 total=100, **bad)
        assert lib.cxs_compressed_select_nsa(sg, q, None, q, q, q, None, None) == \
            _lib.ERR_INVALID
    sg = _lib.SelectGeometry(queries=1, heads=2, block_size=64, count=16, summaries=1039,
                             window=32, stride=16, total=16640)
    columns = _lib.c_i32(0)
    assert lib.cxs_select_score_columns(sg, columns) == _lib.OK and columns.value == 260
    sg.window = sg.stride = 64
    assert lib.cxs_select_score_columns(sg, columns) == _lib.OK and columns.value == 1039
    # Window compression: 32-token windows only.
    assert lib.cxs_compress_windows(q, q, 1, 2, 16, 256, q, q, q, q, q, q, None) == \
        _lib.ERR_INVALID
    # Exchange: 2..8 ranks, rank inside.
    peers = (ctypes.c_void_p * 2)(None, 16)
    assert lib.cxs_exchange_barrier(q, peers, q, 0, 1, 100, q, None) == _lib.ERR_INVALID
    assert lib.cxs_exchange_barrier(q, peers, q, 2, 2, 100, q, None) == _lib.ERR_INVALID
    assert lib.cxs_exchange_barrier(q, (ctypes.c_void_p * 2)(None, None), q, 0, 2, 100, q,
                                    None) == _lib.ERR_INVALID


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc required")
def test_noalloc_limit_matches_header(tmp_path):
    """The Python mirror of CXS_NOALLOC_MAX_PHYSICAL is the header's value."""
    c_file = tmp_path / "limit.c"
    c_file.write_text('#include <stdio.h>\n#include "cxlsparse.h"\n'
                      'int main(void) { printf("%d\\n", CXS_NOALLOC_MAX_PHYSICAL); return 0; }\n')
    exe = tmp_path / "limit"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(c_file), "-o", str(exe)], check=True)
    value = int(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert value == _lib.NOALLOC_MAX_PHYSICAL
    assert _lib.NOALLOC_SCRATCH_BYTES == 16 * value + 256
