"""Window branch and gate fusion inside the fetch/attend launch."""

import pytest
import torch

from cxlsparse_b200.transport import GRSelectedTransport
from nsa_case import setup_case
from oracle import attention as A

pytestmark = pytest.mark.gpu


def _window_case(window, extend, start=0, seed=9):
    g = torch.Generator().manual_seed(seed)
    records = torch.randn(window - 1 + extend, 2, 128, generator=g).bfloat16()
    return records


@pytest.mark.parametrize("window", [16, 64, 128])
def test_window_branch_and_gate_mix(cuda, window):
    pool, cache, backing, query, positions, blocks, fetches = setup_case("partial")
    # Window buffer: the retained history tail + this call's suffix KV.
    saved = min(window - 1, 67)
    records = backing[67 - saved:].contiguous()
    window_start = 67 - saved
    g = torch.Generator().manual_seed(5)
    compressed = torch.randn(13, 2, 16, 64, generator=g).bfloat16()
    gates = torch.rand(13, 2, 16, 3, generator=g).bfloat16()
    transport = GRSelectedTransport(cache, hot_policy="static")
    try:
        for trick, gate in (("window", (0.0, 0.0, 1.0)), ("selected", (0.0, 1.0, 0.0)),
                            ("compressed", (1.0, 0.0, 0.0)), ("mix", None)):
            gt = gates if gate is None else torch.tensor(gate).bfloat16().expand(13, 2, 16, 3)
            out, _ = transport.run(query, blocks, positions, fetches, 16, window=window,
                                   window_kv=records.cuda(), window_start=window_start,
                                   compressed=compressed.cuda(), gates=gt.contiguous().cuda())
            torch.cuda.synchronize()
            out = out.cpu().float()
            win = A.window_attention(query.cpu().float(), records.float(), positions.cpu(),
                                     window_start, window)
            sel = A.selected_attention(query.cpu(), backing, blocks.cpu(), positions.cpu(), 16)
            if trick == "window":
                torch.testing.assert_close(out, win, rtol=0.03, atol=0.03)
            elif trick == "selected":
                torch.testing.assert_close(out, sel.float(), rtol=0.03, atol=0.03)
            elif trick == "compressed":
                assert torch.equal(out, compressed.float())
            else:
                expected = A.gate_mix(sel.bfloat16(), compressed, win.bfloat16(), gt)
                torch.testing.assert_close(out, expected.float(), rtol=0.03, atol=0.03)
    finally:
        transport.close()
        pool.close()
