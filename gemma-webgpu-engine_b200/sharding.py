"""Multi-GPU sampling: one process per GPU, torch.distributed for the plumbing.

Two layouts (the reference samples one row on one device, src/runtime/sampling.ts:18;
these are the B200 deployment of the same call):

* row-sharded (large batches, e.g. C4): contiguous row blocks per rank, each rank runs
  ``GpuSampler.sample`` on its block; there is no collective on the data path.  The ids
  come back to every rank with one all-gather when the caller wants them there.
* vocabulary-sharded (small batches, e.g. C5): every rank holds a slice of every row's
  logits; ``GpuSampler.shard_partials`` streams the slice into a fixed-size record per row,
  one all-gather exchanges the records, and ``GpuSampler.shard_merge`` samples from them,
  identically on every rank.  ``NcclShardedSampler`` does the same step with the
  library's own NCCL exchange (gs_shard_sample), for hosts without a framework collective.

The partition rules and the exchange are plain host logic (tested with gloo on CPU);
the device work is the library's.
"""
from __future__ import annotations

from dataclasses import dataclass

VOCAB_GRANULE = 4096  # shard starts are multiples of this many ids (TMA-aligned mask words)


def row_shards(rows: int, world: int) -> list:
    """(start, count) of each rank's contiguous row block; the first ``rows % world``
    ranks take one extra row."""
    if rows < 0 or world < 1:
        raise ValueError("rows >= 0 and world >= 1")
    base, extra = divmod(rows, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, n))
        start += n
    return out


def vocab_shards(vocab: int, world: int, granule: int = VOCAB_GRANULE) -> list:
    """(offset, size) of each rank's vocabulary slice: equal slices rounded to whole
    granules, the last rank taking the remainder (every offset a multiple of ``granule``)."""
    if vocab <= 0 or world < 1:
        raise ValueError("vocab > 0 and world >= 1")
    per = -(-vocab // world)
    per = -(-per // granule) * granule
    out = []
    for r in range(world):
        off = min(r * per, vocab)
        out.append((off, max(0, min(per, vocab - off))))
    if any(size == 0 for _, size in out):
        raise ValueError(f"vocabulary {vocab} too small for {world} shards of {granule}-id granules")
    return out


def exchange_records(local, group=None):
    """All-gathers each rank's record buffer (a contiguous uint8 tensor of equal size on
    every rank) into one tensor in rank order: [world * local.numel()] bytes, i.e.
    [shards][rows][record] for shard records.  NCCL for CUDA tensors, gloo for CPU."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = local.reshape(-1).contiguous()
    out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    if flat.device.type == "cuda":
        dist.all_gather_into_tensor(out, flat, group=group)
    else:
        parts = list(out.view(world, -1).unbind(0))
        dist.all_gather(parts, flat, group=group)
    return out


def gather_rows(local, rows_total: int, group=None):
    """Row-sharded results (``local`` = this rank's block of a per-row tensor, blocks laid
    out by ``row_shards``) gathered on every rank into [rows_total, ...]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    shards = row_shards(rows_total, world)
    width = max(n for _, n in shards)
    tail = tuple(local.shape[1:])
    pad = torch.zeros((width,) + tail, dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    flat = exchange_records(pad.view(torch.uint8) if pad.dtype != torch.uint8 else pad, group)
    blocks = flat.view(world, -1).view(pad.dtype).view((world, width) + tail)
    return torch.cat([blocks[r, :n] for r, (_, n) in enumerate(shards)], dim=0)


@dataclass
class ShardPlan:
    rank: int
    world: int
    vocab_total: int
    offset: int
    size: int


class VocabShardedSampler:
    """Vocabulary-sharded sampling over ``torch.distributed`` (one process per GPU)."""

    def __init__(self, sampler, vocab_total: int, group=None):
        import torch.distributed as dist
        self.sampler = sampler
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        off, size = vocab_shards(vocab_total, world)[rank]
        self.plan = ShardPlan(rank, world, vocab_total, off, size)

    def sample(self, local_logits, params, *, softcap: float = 0.0, history=None, history_len=None,
               mask_table=None, mask_state=None, rng_state=None, uniforms=None, logprob: bool = False,
               candidates: int = 0, stream=None):
        """``local_logits`` [rows, plan.size] holds this rank's slice; the other arguments
        are the whole rows' (global history ids, full mask table, per-row PRNG states:
        every rank advances its copy identically)."""
        p = self.plan
        if local_logits.shape[1] != p.size:
            raise ValueError(f"rank {p.rank} holds {p.size} ids, got {local_logits.shape[1]}")
        rec = self.sampler.shard_partials(local_logits, params, vocab_offset=p.offset, vocab_total=p.vocab_total,
                                          softcap=softcap, history=history, history_len=history_len,
                                          mask_table=mask_table, mask_state=mask_state, logprob=logprob,
                                          stream=stream)
        gathered = exchange_records(rec, self.group)
        hstride = 0 if history is None else (history.stride(0) if history.shape[0] > 1 else history.shape[1])
        return self.sampler.shard_merge(gathered, params, rows=local_logits.shape[0], shards=p.world,
                                        vocab_total=p.vocab_total, history_stride=hstride, mask_table=mask_table,
                                        mask_state=mask_state, rng_state=rng_state, uniforms=uniforms,
                                        logprob=logprob, candidates=candidates, stream=stream)


class NcclShardedSampler:
    """Vocabulary-sharded sampling with the library's own NCCL exchange (gs_nccl_create +
    gs_shard_sample): the same result as ``VocabShardedSampler`` without a framework
    collective, the form an addon without torch binds.  Every rank constructs it with the
    same ``unique_id`` (made once by ``NcclShardedSampler.unique_id()`` and sent to the
    others by any means).  A rank that never joins ends set-up or a step with
    ``SamplerError`` (GS_ETIMEOUT) after ``timeout_ms``; the communicator is then aborted and
    a new sampler is needed."""

    def __init__(self, sampler, vocab_total: int, rank: int, world: int, unique_id: bytes, timeout_ms: int = 30000):
        import ctypes
        from . import _lib
        from .sampling import SamplerError
        self._L = _lib.lib()
        self._lib = _lib
        self.sampler = sampler
        self.timeout_ms = int(timeout_ms)
        off, size = vocab_shards(vocab_total, world)[rank]
        self.plan = ShardPlan(rank, world, vocab_total, off, size)
        if len(unique_id) != 128:
            raise ValueError("the communicator id is 128 bytes")
        idb = (ctypes.c_char * 128).from_buffer_copy(unique_id)
        self._comm = ctypes.c_void_p()
        st = self._L.gs_nccl_create(sampler.device, idb, world, rank, self.timeout_ms, ctypes.byref(self._comm))
        if st != _lib.GS_OK:
            raise SamplerError(st, (self._L.gs_nccl_last_error(None) or b"").decode())

    @staticmethod
    def unique_id() -> bytes:
        import ctypes
        from . import _lib
        from .sampling import SamplerError
        L = _lib.lib()
        idb = (ctypes.c_char * 128)()
        st = L.gs_nccl_unique_id(idb)
        if st != _lib.GS_OK:
            raise SamplerError(st, (L.gs_nccl_last_error(None) or b"").decode())
        return bytes(idb)

    def sample(self, local_logits, params, *, softcap: float = 0.0, history=None, history_len=None, mask_table=None,
               mask_state=None, rng_state=None, uniforms=None, logprob: bool = False, candidates: int = 0,
               stream=None):
        """``local_logits`` [rows, plan.size] is this rank's slice; the other arguments are
        the whole rows' (as ``VocabShardedSampler.sample``).  Asynchronous on ``stream``
        unless ``timeout_ms`` > 0, when the call waits for the step (bounded)."""
        import ctypes
        import torch
        from .sampling import SamplerError
        p = self.plan
        if local_logits.shape[1] != p.size:
            raise ValueError(f"rank {p.rank} holds {p.size} ids, got {local_logits.shape[1]}")
        s = self.sampler
        b, keep = s.make_batch(local_logits, params, softcap=softcap, history=history, history_len=history_len,
                               mask_table=mask_table, mask_state=mask_state, rng_state=rng_state, uniforms=uniforms)
        out, o = s.make_outputs(local_logits.shape[0], local_logits.device, logprob, candidates)
        if stream is None:
            stream = torch.cuda.current_stream(local_logits.device).cuda_stream
        st = self._L.gs_shard_sample(s.handle, self._comm, ctypes.byref(b), p.offset, p.vocab_total, ctypes.byref(o),
                                     self.timeout_ms, ctypes.c_void_p(stream))
        del keep
        if st != self._lib.GS_OK:
            raise SamplerError(st, (self._L.gs_nccl_last_error(self._comm) or b"").decode())
        return out

    def close(self):
        if self._comm:
            self._L.gs_nccl_destroy(self._comm)
            import ctypes
            self._comm = ctypes.c_void_p()
