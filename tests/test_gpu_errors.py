"""Bounded waits end with an error status instead of hanging the GPU.

A missing block whose IO entry is withheld (missing count forced to 0) is
never published: every attention warp that needs it gives up after the spin
limit, records CXS_DEVICE_ERR_READY_TIMEOUT and the launch completes. No GPU
fault, trap or unbounded wait is involved.
"""

import pytest
import torch

from cxlsparse_b200 import _lib
from cxlsparse_b200.transport import GRSelectedTransport
from nsa_case import setup_case

pytestmark = pytest.mark.gpu


def test_unpublished_block_times_out_with_error_status(cuda):
    pool, cache, backing, query, positions, blocks, fetches = setup_case("miss")
    transport = GRSelectedTransport(cache, hot_policy="static", spin_limit=20_000_000)
    try:
        output, counters = transport.run(query, blocks, positions, fetches, 16)
        transport.last_done.synchronize()
        counters.materialize()
        w = transport.workspace()
        assert int(w["missing"].item()) > 0
        stream = torch.cuda.current_stream()
        transport.active_plan.plan(w, stream)
        w["missing"].zero_()  # withhold every IO entry: nothing publishes ready
        geometry = _lib.AttendGeometry(
            queries=w["queries"], heads=w["heads"], width=w["width"], block_size=16,
            physical=w["physical"], spin_limit=20_000_000)
        _lib.check(_lib.lib().cxs_fetch_attend(geometry, w["c_attend_buffers"],
                                               stream.cuda_stream))
        torch.cuda.synchronize()
        assert int(w["error"].item()) & _lib.DEVICE_ERR_READY_TIMEOUT
        # The context stays usable: a normal call afterwards succeeds.
        output, counters = transport.run(query, blocks, positions, fetches, 16)
        transport.last_done.synchronize()
        counters.materialize()
        assert torch.isfinite(output).all()
    finally:
        transport.close()
        pool.close()
