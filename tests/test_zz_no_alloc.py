"""The allocation-free fetch/attend entry point matches the regular one.

cxs_fetch_attend_noalloc serves callers that cannot allocate device memory on
their own (for example a plugin whose host process's allocator owns the whole
GPU, or code that must avoid cudaMalloc's device-wide synchronisation after
start-up): its block-source scratch lives in a fixed static device array of
the library instead of caller buffers. This file is collected last so a
failure here cannot hide earlier results; it also passes alone in a fresh
process.
"""

import pytest
import torch

from cxlsparse_b200 import _lib
from cxlsparse_b200.transport import GRSelectedTransport
from nsa_case import setup_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("residency", ["miss", "partial"])
def test_noalloc_entry_point_matches_regular_entry_point(cuda, residency):
    pool, cache, backing, query, positions, blocks, fetches = setup_case(residency)
    transport = GRSelectedTransport(cache, hot_policy="static")
    try:
        expected, counters = transport.run(query, blocks, positions, fetches, 16)
        transport.last_done.synchronize()
        counters.materialize()
        expected = expected.clone()
        w = transport.workspace()
        geometry = _lib.AttendGeometry(
            queries=w["queries"], heads=w["heads"], width=w["width"], block_size=w["bs"],
            physical=w["physical"], spin_limit=1 << 32)
        out = torch.full_like(w["output"], float("nan"))
        error = torch.full((1,), 7, dtype=torch.int32, device=cuda)
        buffers = _lib.AttendBuffers(**{f: getattr(w["c_attend_buffers"], f)
                                        for f, _ in _lib.AttendBuffers._fields_})
        buffers.out, buffers.error = out.data_ptr(), error.data_ptr()
        buffers.sources = buffers.kinds = buffers.ready = buffers.control = None
        stream = torch.cuda.current_stream()
        for _ in range(2):  # two calls in a row share (and re-initialise) the scratch
            out.fill_(float("nan"))
            _lib.check(_lib.lib().cxs_fetch_attend_noalloc(geometry, buffers,
                                                           stream.cuda_stream))
            torch.cuda.synchronize()
            assert int(error.item()) == 0
            torch.testing.assert_close(out[: len(query)].float(), expected.float(),
                                       rtol=0.03, atol=0.03)
    finally:
        transport.close()
        pool.close()


def test_noalloc_rejects_oversized_geometry(cuda):
    geometry = _lib.AttendGeometry(queries=1, heads=2, width=4, block_size=16,
                                   physical=_lib.NOALLOC_MAX_PHYSICAL + 1)
    buffers = _lib.AttendBuffers()
    status = _lib.lib().cxs_fetch_attend_noalloc(geometry, buffers, None)
    assert status == _lib.ERR_CAPACITY
    assert b"at most" in _lib.lib().cxs_last_error()
