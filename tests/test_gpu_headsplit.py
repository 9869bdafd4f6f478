"""KV-head split across a GPU pair (the long-history serving layout, scaled down).

Rank i of the pair owns KV head i of every layer: its 16 query heads, its own
pool slice, cache rows, planner, fetch and attention; each attention launch
stores its output rows into both GPUs' gather buffers (NVLink stores, CUDA
IPC) and a bounded flag barrier per layer hands them over before o_proj. The
pair's extend must reproduce the single-GPU model that holds both heads,
eagerly and from a captured graph that contains the exchange. Needs two GPUs.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HISTORY, EXTEND, LAYERS = 1000, 64, 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(vocab):
    g = torch.Generator().manual_seed(21)
    return (torch.randint(0, vocab, (HISTORY,), generator=g),
            torch.randint(0, vocab, (EXTEND,), generator=g))


def _rank(rank, port, results):
    import datetime

    import torch.distributed as dist

    from cxlsparse_b200.model import NSAConfig, NSAExtendModel
    from cxlsparse_b200.sharding import PeerExchange, head_pair_groups

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=device,
                            timeout=datetime.timedelta(seconds=120))
    try:
        group, shard, shards, _, _ = head_pair_groups(2)
        cfg = NSAConfig(layers=LAYERS, hot=64)
        # About half a second per wait: a peer that never arrives sets the
        # error word instead of holding the GPU.
        exchange = PeerExchange(group, shard, shards, rows=1024, kv_heads=cfg.kv_heads,
                                kv_local=1, device=device, spin_limit=1 << 30)
        model = NSAExtendModel(cfg, device=device, seed=0, max_history=HISTORY + EXTEND,
                               chunk=512, head_shard=(shard, shards), exchange=exchange)
        history, ids = _inputs(cfg.vocab)
        model.prefill(history.to(device))
        eager = model.extend(ids.to(device)).float().cpu()
        graph, static_ids, static_out, counters = model.capture_extend(EXTEND)
        static_ids.copy_(ids.to(device))
        graph.replay()
        torch.cuda.synchronize()
        misses = sum(r[0]["misses"] for c in counters for r in [c.materialize()])
        exchange.check()
        results[rank] = (eager, static_out.float().cpu(), misses)
        del graph
        model.close()
        exchange.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_head_pair_matches_single_gpu_model(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from cxlsparse_b200.model import NSAConfig, NSAExtendModel

    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_rank, args=(_port(), results), nprocs=2, start_method="spawn")
    cfg = NSAConfig(layers=LAYERS, hot=64)
    full = NSAExtendModel(cfg, device=cuda, seed=0, max_history=HISTORY + EXTEND, chunk=512)
    try:
        history, ids = _inputs(cfg.vocab)
        full.prefill(history.to(cuda))
        expected = full.extend(ids.to(cuda)).float().cpu()
    finally:
        full.close()
    for rank in (0, 1):
        eager, graphed, misses = results[rank]
        assert misses > 0
        torch.testing.assert_close(eager, expected, rtol=0.02, atol=0.02)
        torch.testing.assert_close(graphed, expected, rtol=0.02, atol=0.02)
    assert torch.equal(results[0][0], results[1][0])  # both ranks hold the same hidden states
