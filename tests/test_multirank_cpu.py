"""Multi-rank host logic on CPU with gloo (world size 2): row shards of
128-row chunks reassemble the unsharded Q and S byte for byte, the timing
reduction takes the max over ranks, and a rank that leaves before the
barrier makes the others fail within the process-group timeout."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import MXFP8_quantizer

shard = MXFP8_quantizer.load_package().shard


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, m, k, result_q):
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(__file__)))
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "oracle"))
    import inputs
    import oracle

    _init(rank, world, port)
    bits = inputs.normal(m, k, 123, "bf16")
    r0, r1 = shard.row_shard(m, world, rank)
    q, s = oracle.quantize(bits[r0:r1], "bf16", r1 - r0, k)
    b0, b1 = shard.scale_byte_range(r0, r1, k)
    assert s.size == b1 - b0
    # gather variable-size shards: pad to the largest
    qmax = m * k
    smax = oracle.scale_storage_bytes(m, k)
    qt = torch.zeros(qmax, dtype=torch.uint8)
    qt[: q.size] = torch.from_numpy(q.reshape(-1))
    st = torch.zeros(smax, dtype=torch.uint8)
    st[: s.size] = torch.from_numpy(s)
    qs = [torch.zeros_like(qt) for _ in range(world)]
    ss = [torch.zeros_like(st) for _ in range(world)]
    dist.all_gather(qs, qt)
    dist.all_gather(ss, st)
    slowest = shard.max_over_ranks(float(rank + 1))
    if rank == 0:
        q_full, s_full = oracle.quantize(bits, "bf16", m, k)
        parts_q, parts_s = [], []
        for r in range(world):
            a0, a1 = shard.row_shard(m, world, r)
            c0, c1 = shard.scale_byte_range(a0, a1, k)
            parts_q.append(qs[r][: (a1 - a0) * k].numpy())
            parts_s.append(ss[r][: c1 - c0].numpy())
        ok = (np.array_equal(np.concatenate(parts_q), q_full.reshape(-1))
              and np.array_equal(np.concatenate(parts_s), s_full) and slowest == float(world))
        result_q.put(ok)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("m", [640, 1000])
def test_row_shards_reassemble_unsharded_output(m):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_shard_worker, args=(2, free_port(), m, 544, q), nprocs=2, join=True,
                       start_method="spawn")
    assert q.get() is True


def _leaver_worker(rank, world, port, result_q):
    _init(rank, world, port, timeout_s=3)
    if rank == 1:
        return  # leaves between steps, without joining the barrier
    try:
        dist.barrier()
        result_q.put("no error")
    except Exception as exc:  # the process-group timeout ends the wait
        result_q.put(type(exc).__name__)


def test_rank_that_leaves_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_leaver_worker, args=(2, free_port(), q), nprocs=2, join=True, start_method="spawn")
    assert q.get() != "no error"


def test_row_shard_arithmetic():
    for m in (1, 127, 128, 129, 8192, 16384 * 8 + 5):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.row_shard(m, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == m
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            for a0, a1 in spans:
                assert a0 % 128 == 0 or a0 == a1 == m   # empty trailing shards start at m
    assert shard.row_shard(8192 * 8, 8, 3) == (3 * 8192, 4 * 8192)
    assert shard.scale_byte_range(128, 256, 8192) == (64 * 512, 2 * 64 * 512)  # 64 chunks per row block
