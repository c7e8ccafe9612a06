"""Multi-process host logic of the multi-GPU layouts, on CPU: gloo, world_size 2.

The device work (partials, merge) is covered by the GPU tests; here the partition rules,
the record exchange order and the row gather run as real torch.distributed ranks.
"""
from __future__ import annotations

import importlib
import os
import socket

import pytest

SH = importlib.import_module("gemma-webgpu-engine_b200.sharding")


def test_row_shards_cover_rows():
    for rows in (0, 1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            sh = SH.row_shards(rows, world)
            assert len(sh) == world
            assert sum(n for _, n in sh) == rows
            start = 0
            for s, n in sh:
                assert s == start and n >= 0
                start += n
            assert max(n for _, n in sh) - min(n for _, n in sh) <= 1


def test_vocab_shards_aligned_and_disjoint():
    for vocab, world in ((262144, 8), (262144, 2), (262144, 3), (50000, 4), (4096, 1)):
        sh = SH.vocab_shards(vocab, world)
        assert sh[0][0] == 0
        for (o, n), (o2, _) in zip(sh, sh[1:]):
            assert o % SH.VOCAB_GRANULE == 0 and o + n == o2
        assert sh[-1][0] + sh[-1][1] == vocab
    assert SH.vocab_shards(262144, 8) == [(32768 * g, 32768) for g in range(8)]
    with pytest.raises(ValueError):
        SH.vocab_shards(4096, 2)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    sh = importlib.import_module("gemma-webgpu-engine_b200.sharding")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        # shard records: rank r, row i, byte j = 100*r + 10*i + j
        rows, rec = 3, 5
        local = torch.tensor([[100 * rank + 10 * i + j for j in range(rec)] for i in range(rows)],
                             dtype=torch.uint8)
        got = sh.exchange_records(local)
        torch.save(got, os.path.join(out_dir, f"records_{rank}.pt"))
        # row gather: 5 rows over 2 ranks (blocks of 3 and 2), ids = global row * 7
        total = 5
        start, n = sh.row_shards(total, world)[rank]
        ids = torch.arange(start, start + n, dtype=torch.int32) * 7
        torch.save(sh.gather_rows(ids, total), os.path.join(out_dir, f"rows_{rank}.pt"))
        # 2-D per-row results (e.g. candidate lists) keep their trailing shape
        cand = torch.stack([torch.arange(4, dtype=torch.float64) + 10 * r for r in range(start, start + n)])
        torch.save(sh.gather_rows(cand, total), os.path.join(out_dir, f"cands_{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_exchange_and_gather_two_ranks(tmp_path):
    import torch
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    rows, rec = 3, 5
    want = torch.tensor([[100 * r + 10 * i + j for j in range(rec)] for r in range(2) for i in range(rows)],
                        dtype=torch.uint8).reshape(-1)
    for r in range(2):
        assert torch.equal(torch.load(tmp_path / f"records_{r}.pt"), want), f"rank {r} record order"
        assert torch.load(tmp_path / f"rows_{r}.pt").tolist() == [7 * i for i in range(5)]
        c = torch.load(tmp_path / f"cands_{r}.pt")
        assert c.shape == (5, 4)
        assert torch.equal(c, torch.stack([torch.arange(4, dtype=torch.float64) + 10 * i for i in range(5)]))
