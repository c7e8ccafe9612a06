"""Vocabulary-sharded mode (gs_shard_partials -> all-gather -> gs_shard_merge) on GPU.

One GPU plays every shard (the records are concatenated in shard order, as the
all-gather lays them out); the merged result must match the oracle on the whole rows and
gs_sample on the whole rows.  A two-process NCCL run covers the real exchange when two
GPUs are visible.
"""
from __future__ import annotations

import importlib
import os
import socket

import numpy as np
import pytest

import parity_util as PU

pytestmark = pytest.mark.gpu


def _shards_run(sampler, x, p, shards, *, softcap=30.0, hist=None, hlen=None, table=None, mstate=None, uniforms,
                logprob=False, cand=2048):
    import torch
    SH = importlib.import_module("gemma-webgpu-engine_b200.sharding")
    dev = torch.device("cuda", 0)
    V = x.shape[1]
    xt = torch.from_numpy(x).to(dev)
    ht = None if hist is None else torch.from_numpy(hist).to(dev)
    hl = None if hlen is None else torch.from_numpy(hlen).to(dev)
    tt = None if table is None else torch.from_numpy(table.view(np.int32)).to(dev)
    mt = None if mstate is None else torch.from_numpy(mstate).to(dev)
    recs = []
    for off, size in SH.vocab_shards(V, shards):
        recs.append(sampler.shard_partials(xt[:, off:off + size].contiguous(), [p], vocab_offset=off, vocab_total=V,
                                           softcap=softcap, history=ht, history_len=hl, mask_table=tt,
                                           mask_state=mt, logprob=logprob))
    gathered = torch.cat([r.reshape(-1) for r in recs])
    u = torch.from_numpy(uniforms).to(dev)
    res = sampler.shard_merge(gathered, [p], rows=x.shape[0], shards=shards, vocab_total=V,
                              history_stride=0 if hist is None else hist.shape[1], mask_table=tt, mask_state=mt,
                              uniforms=u, logprob=logprob, candidates=cand)
    torch.cuda.synchronize()
    return PU.GpuOut(ids=res.ids.cpu().numpy(), flags=res.flags.cpu().numpy().view(np.uint32), rng_after=None,
                     cand_ids=res.cand_ids.cpu().numpy(), cand_probs=res.cand_probs.cpu().numpy(),
                     cand_count=res.cand_count.cpu().numpy(),
                     logprob=None if res.logprob is None else res.logprob.cpu().numpy())


def _c5_rows(rows=8, V=262144, seed=41):
    rng = np.random.default_rng(seed)
    u = rng.random((rows, V)).clip(1e-300, 1 - 1e-16)
    x = (-2.0 * np.log(-np.log(u))).astype(np.float32)
    for r in range(rows):  # 30 planted exact ties at the row maximum
        x[r, rng.choice(V, 30, replace=False)] = x[r].max()
    return x


def test_c5_vocab_sharded_matches_oracle_and_whole_rows(oracle, sampler):
    """C5: 8 rows, 8 shards of 32768 ids, topK 1024, T 1.5, P 0.99, planted ties."""
    x = _c5_rows()
    p = {"temperature": 1.5, "topK": 1024, "topP": 0.99, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
         "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
    u = np.random.default_rng(7).random(8)
    got = _shards_run(sampler, x, p, 8, softcap=30.0, uniforms=u)
    ids, margins, cands, _ = PU.oracle_rows(oracle, x, x.shape[1], 30.0, [p], uniforms=u)
    PU.compare(got, ids, margins, cands, label="c5-sharded")
    whole = PU.run_gpu(sampler, x, [p], softcap=30.0, uniforms=u)
    assert (got.ids == whole.ids).all() or (got.flags & pkg_flag_boundary()).any()
    np.testing.assert_array_equal(got.cand_count, whole.cand_count)


def pkg_flag_boundary():
    return importlib.import_module("gemma-webgpu-engine_b200")._lib.FLAG_BOUNDARY


@pytest.mark.parametrize("k,temp,logprob", [(50, 0.8, True), (1, 0.0, False), (64, 0.7, False)],
                         ids=["k50-logprob", "greedy", "k64"])
def test_sharded_with_history_and_mask(oracle, sampler, k, temp, logprob):
    """Penalised ids and constrained rows across 4 shards (the history ids and the mask
    bits are global; each shard scores the penalised ids it holds)."""
    rng = np.random.default_rng(300 + k)
    V, rows, H = 65536, 10, 300
    x = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
    dens = [0.01, 0.05, 0.3, 1.0]
    allowed = rng.random((len(dens), V)) < np.array(dens)[:, None]
    allowed[:, 5] = True
    bits = allowed.reshape(len(dens), V // 32, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    table = bits.sum(axis=-1).astype(np.uint32)
    mstate = np.array([(i % (len(dens) + 1)) - 1 for i in range(rows)], dtype=np.int32)
    hist = np.zeros((rows, H), dtype=np.int32)
    hlen = np.zeros(rows, dtype=np.int32)
    for r in range(rows):
        h = rng.integers(0, V, H) if r % 2 else rng.choice(20000, H, replace=False)
        hist[r] = h
        hlen[r] = H
    p = {"temperature": temp, "topK": k, "topP": 0.95, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.2,
         "presencePenalty": 0.4, "frequencyPenalty": 0.2, "repetitionWindow": H}
    u = rng.random(rows)
    got = _shards_run(sampler, x, p, 4, hist=hist, hlen=hlen, table=table, mstate=mstate, uniforms=u,
                      logprob=logprob)
    ids, margins, cands, _ = PU.oracle_rows(oracle, x, V, 30.0, [p], history=hist, history_len=hlen,
                                            mask_table=table, mask_state=mstate, uniforms=u)
    assert PU.compare(got, ids, margins, cands, label=f"sharded-k{k}") <= 1
    if logprob:
        for r in range(rows):
            ref = oracle.token_log_probability(oracle.softcap(x[r], 30.0), int(got.ids[r]))
            assert abs(got.logprob[r] - ref) <= 1e-6 * max(1.0, abs(ref)), r


def test_sharded_rejects_full_vocabulary_topk(sampler):
    import torch
    pkg = importlib.import_module("gemma-webgpu-engine_b200")
    x = torch.zeros((2, 4096), device="cuda")
    p = {"temperature": 1.0, "topK": 0, "topP": 0.9, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
         "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
    with pytest.raises(pkg.SamplerError, match="vocabulary-sharded mode needs"):
        sampler.shard_partials(x, p, vocab_offset=0, vocab_total=8192)
    p["topK"] = 10
    with pytest.raises(ValueError, match="multiple of 4096"):
        sampler.shard_partials(x, p, vocab_offset=100, vocab_total=8192)


# ----------------------------------------------------------------- two GPUs, real NCCL

def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_worker(rank, world, port, out_dir):
    import datetime
    import torch
    import torch.distributed as dist
    pkg = importlib.import_module("gemma-webgpu-engine_b200")
    SH = importlib.import_module("gemma-webgpu-engine_b200.sharding")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        x = torch.from_numpy(_c5_rows(rows=8, V=262144)).to(dev)
        p = {"temperature": 1.5, "topK": 1024, "topP": 0.99, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
             "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
        sampler = pkg.GpuSampler(rank)
        vs = SH.VocabShardedSampler(sampler, 262144)
        off, size = vs.plan.offset, vs.plan.size
        rng = torch.tensor([pkg.SeededRandom(4000 + i).state for i in range(8)], dtype=torch.float64, device=dev)
        res = vs.sample(x[:, off:off + size].contiguous(), [p], softcap=30.0, rng_state=rng, candidates=64)
        torch.cuda.synchronize()
        torch.save({"ids": res.ids.cpu(), "rng": rng.cpu(), "cand": res.cand_ids.cpu()},
                   os.path.join(out_dir, f"nccl_{rank}.pt"))
        sampler.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_nccl_exchange(tmp_path, sampler):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(NCCL_NVLS_ENABLE="0")
    os.environ.update(env)
    mp.start_processes(_nccl_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    pkg = importlib.import_module("gemma-webgpu-engine_b200")
    x = torch.from_numpy(_c5_rows(rows=8, V=262144)).cuda()
    p = {"temperature": 1.5, "topK": 1024, "topP": 0.99, "minP": 0.0, "typicalP": 1.0, "repetitionPenalty": 1.0,
         "presencePenalty": 0.0, "frequencyPenalty": 0.0, "repetitionWindow": 0}
    rng = torch.tensor([pkg.SeededRandom(4000 + i).state for i in range(8)], dtype=torch.float64, device="cuda")
    whole = sampler.sample(x, [p], softcap=30.0, rng_state=rng, candidates=64)
    torch.cuda.synchronize()
    r0, r1 = (torch.load(tmp_path / f"nccl_{r}.pt") for r in range(2))
    assert torch.equal(r0["ids"], r1["ids"]) and torch.equal(r0["rng"], r1["rng"])
    assert torch.equal(r0["rng"], rng.cpu())
    flags = whole.flags.cpu().numpy().view(np.uint32)
    same = (r0["ids"] == whole.ids.cpu()).numpy()
    assert (same | ((flags & pkg._lib.FLAG_BOUNDARY) != 0)).all()
