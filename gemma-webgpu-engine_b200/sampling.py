"""Host-side mirror of the reference sampler interface, backed by libgsampler (CUDA).

Reference interface (aribornstein/gemma-webgpu-engine, src/runtime/sampling.ts):
  SeededRandom(seed).next()                          :3-16
  sampleToken(rawLogits, history, config, random)    :18-65
  tokenLogProbability(rawLogits, token)              :67-80
and src/runtime/constraints.ts:159-173 maskConstraintLogits.

The functions keep the reference's names (snake_case), argument meaning and error
messages.  Sampling itself always runs on the GPU through the C ABI; torch is used only
to hold device buffers.  There is no CPU fallback: without libgsampler.so or a CUDA
device every call raises.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np

from . import _lib
from ._lib import GsBatch, GsOutputs, GsParams

# ----------------------------------------------------------------------------- errors


class SamplerError(RuntimeError):
    """A libgsampler call failed; ``status`` is the gs_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _raise(status: int, ctx, what: str = ""):
    msg = ""
    if ctx is not None:
        raw = _lib.lib().gs_last_error(ctx)
        msg = raw.decode() if raw else ""
    if status == _lib.GS_EEMPTY:
        raise ValueError("Cannot sample empty logits")
    if status == _lib.GS_EDEADEND:
        raise SamplerError(status, "Generation constraint reached a tokenization dead end")
    if status == _lib.GS_EINVAL:
        raise ValueError(msg or what)
    raise SamplerError(status, msg or what or f"libgsampler status {status}")


# ----------------------------------------------------------------------- SeededRandom


class SeededRandom:
    """Mulberry32 over a JS-number state (src/runtime/sampling.ts:3-16).

    ``state`` is the same double the reference keeps; the GPU path reads and advances it
    (one draw per sampled row), so a stream can move between host and device freely.
    """

    def __init__(self, seed: float):
        s = int(math.trunc(seed)) % 4294967296
        self.state = float(s) if s != 0 else float(0x6D2B79F5)

    def next(self) -> float:
        self.state = self.state + 1831565813.0
        v = int(math.fmod(self.state, 4294967296.0)) & 0xFFFFFFFF
        v = ((v ^ (v >> 15)) * (v | 1)) & 0xFFFFFFFF
        v ^= (v + ((v ^ (v >> 7)) * (v | 61))) & 0xFFFFFFFF
        v &= 0xFFFFFFFF
        return ((v ^ (v >> 14)) & 0xFFFFFFFF) / 4294967296.0

    def __call__(self) -> float:
        return self.next()


# --------------------------------------------------------------------------- sampler


def params_from_config(config: dict) -> GsParams:
    """The DecodingConfig fields sampleToken reads (src/runtime/decoding.ts:1-14)."""
    top_k = config["topK"]
    return GsParams(float(config["temperature"]), float(config["topP"]), float(config["minP"]),
                    float(config["typicalP"]), float(config["repetitionPenalty"]),
                    float(config["presencePenalty"]), float(config["frequencyPenalty"]),
                    int(top_k) if top_k < 2**31 else 2**31 - 1, 0)


_PARAMS_DTYPE = None


def _params_dtype():
    global _PARAMS_DTYPE
    if _PARAMS_DTYPE is None:
        import numpy as np
        _PARAMS_DTYPE = np.dtype([(n, np.float64) for n in ("temperature", "top_p", "min_p", "typical_p",
                                                            "repetition_penalty", "presence_penalty",
                                                            "frequency_penalty")] +
                                 [("top_k", np.int32), ("reserved", np.int32)])
        assert _PARAMS_DTYPE.itemsize == ctypes.sizeof(GsParams)
    return _PARAMS_DTYPE


def prepare_params(params):
    """The gs_params array of ``params`` (a config dict, a GsParams, or a list of them, one
    per row).  Every sampling call accepts the returned array in place of the list, so a
    decode loop whose per-row configs stay fixed converts them once instead of per step."""
    if isinstance(params, ctypes.Array):
        return params
    if isinstance(params, (dict, GsParams)):
        params = [params]
    if all(isinstance(p, dict) for p in params):
        import numpy as np
        keys = ("temperature", "topP", "minP", "typicalP", "repetitionPenalty", "presencePenalty",
                "frequencyPenalty")
        rec = np.empty(len(params), dtype=_params_dtype())
        for i, k in enumerate(keys):
            rec[rec.dtype.names[i]] = [p[k] for p in params]
        rec["top_k"] = np.minimum(np.array([p["topK"] for p in params], dtype=np.int64), 2**31 - 1)
        rec["reserved"] = 0
        return (GsParams * len(params)).from_buffer(rec)
    return (GsParams * len(params))(*[p if isinstance(p, GsParams) else params_from_config(p) for p in params])


_params_array = prepare_params


def compact_history(history: Sequence[int]) -> tuple[list, list]:
    """A window as its distinct ids in order of first occurrence and the number of times
    each occurs: the form ``history`` + ``history_count`` take.  The penalties depend only
    on each id's count in the window (src/runtime/sampling.ts:21-30), so a window longer
    than MAX_HISTORY entries samples the same way in this form."""
    counts: dict = {}
    for t in history:
        t = int(t)
        counts[t] = counts.get(t, 0) + 1
    return list(counts.keys()), list(counts.values())


def windowed_history(history: Sequence[int], window: int) -> list:
    """history.slice(-config.repetitionWindow), or [] for a zero window (sampling.ts:22-24)."""
    if window == 0:
        return []
    return list(history[-window:]) if window < len(history) else list(history)


@dataclass
class SampleResult:
    ids: object            # [rows] int32 token ids (-1 on a row error)
    flags: object          # [rows] uint32 GS_FLAG_* bits (as int32)
    logprob: object = None
    cand_ids: object = None
    cand_probs: object = None
    cand_count: object = None


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


class GpuSampler:
    """A libgsampler context on one CUDA device (device memory held in torch tensors)."""

    def __init__(self, device: int = 0):
        self.device = device
        self._L = _lib.lib()
        self._ctx = ctypes.c_void_p()
        st = self._L.gs_create(device, ctypes.byref(self._ctx))
        if st != _lib.GS_OK:
            raise SamplerError(st, f"gs_create(device={device}) failed with status {st}")

    @property
    def handle(self):
        return self._ctx

    def close(self):
        if self._ctx:
            self._L.gs_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, rows: int, vocab: int, max_top_k: int, history_stride: int):
        st = self._L.gs_reserve(self._ctx, rows, vocab, max_top_k, history_stride)
        if st != _lib.GS_OK:
            _raise(st, self._ctx)

    def last_error(self) -> str:
        raw = self._L.gs_last_error(self._ctx)
        return raw.decode() if raw else ""

    def make_batch(self, logits, params, *, softcap: float = 0.0, history=None, history_len=None,
                   mask_table=None, mask_state=None, rng_state=None, uniforms=None, history_count=None):
        import torch
        if logits.dim() != 2:
            raise ValueError("logits must be [rows, vocab]")
        if logits.dtype == torch.float32:
            dtype = _lib.GS_DTYPE_F32
        elif logits.dtype == torch.bfloat16:
            dtype = _lib.GS_DTYPE_BF16
        else:
            raise ValueError("logits must be float32 or bfloat16")
        if logits.stride(1) != 1:
            raise ValueError("logits rows must be contiguous")
        rows, vocab = logits.shape
        parr = _params_array(params)
        b = GsBatch()
        b.logits = logits.data_ptr()
        b.dtype = dtype
        b.rows = rows
        b.vocab = vocab
        b.row_stride = logits.stride(0) if rows > 1 else vocab
        b.softcap = float(softcap)
        b.params_count = len(parr)
        b.params = ctypes.cast(parr, ctypes.c_void_p)
        if history is not None:
            b.history = history.data_ptr()
            b.history_len = history_len.data_ptr()
            b.history_stride = history.stride(0) if history.shape[0] > 1 else history.shape[1]
            if history_count is not None:
                if history_count.dtype != torch.int32 or tuple(history_count.shape) != tuple(history.shape) or \
                        history_count.stride() != history.stride():
                    raise ValueError("history_count must be int32 with the history's shape and strides")
                b.history_count = history_count.data_ptr()
        elif history_count is not None:
            raise ValueError("history_count needs a history")
        if mask_table is not None:
            b.mask_table = mask_table.data_ptr()
            b.mask_states = mask_table.shape[0]
            b.mask_words = mask_table.stride(0) if mask_table.shape[0] > 1 else mask_table.shape[1]
            b.mask_state = mask_state.data_ptr()
        if rng_state is not None:
            b.rng_state = rng_state.data_ptr()
        if uniforms is not None:
            b.uniforms = uniforms.data_ptr()
        return b, parr

    @staticmethod
    def make_outputs(rows: int, dev, logprob: bool = False, candidates: int = 0, out: SampleResult | None = None):
        """(SampleResult of device tensors, the gs_outputs pointing at them)."""
        import torch
        if out is None:
            out = SampleResult(
                ids=torch.empty(rows, dtype=torch.int32, device=dev),
                flags=torch.empty(rows, dtype=torch.int32, device=dev),
                logprob=torch.empty(rows, dtype=torch.float64, device=dev) if logprob else None,
                cand_ids=torch.empty((rows, candidates), dtype=torch.int32, device=dev) if candidates else None,
                cand_probs=torch.empty((rows, candidates), dtype=torch.float64, device=dev) if candidates else None,
                cand_count=torch.empty(rows, dtype=torch.int32, device=dev) if candidates else None,
            )
        o = GsOutputs()
        o.ids = _ptr(out.ids)
        o.flags = _ptr(out.flags)
        o.logprob = _ptr(out.logprob)
        o.cand_ids = _ptr(out.cand_ids)
        o.cand_probs = _ptr(out.cand_probs)
        o.cand_count = _ptr(out.cand_count)
        o.cand_cap = out.cand_ids.shape[1] if out.cand_ids is not None else 0
        return out, o

    def sample(self, logits, params, *, softcap: float = 0.0, history=None, history_len=None, mask_table=None,
               mask_state=None, rng_state=None, uniforms=None, logprob: bool = False, candidates: int = 0,
               stream=None, out: SampleResult | None = None, history_count=None) -> SampleResult:
        """Batched sampling of device-resident logits [rows, vocab] (gs_sample).  Asynchronous on
        ``stream`` (torch's current stream when None); outputs are device tensors.
        ``history_count`` (int32, the history's shape): the occurrences each history entry
        stands for (a window given as ``compact_history``'s distinct ids and counts)."""
        import torch
        b, keep = self.make_batch(logits, params, softcap=softcap, history=history, history_len=history_len,
                                  mask_table=mask_table, mask_state=mask_state, rng_state=rng_state,
                                  uniforms=uniforms, history_count=history_count)
        dev = logits.device
        out, o = self.make_outputs(logits.shape[0], dev, logprob, candidates, out)
        if stream is None:
            stream = torch.cuda.current_stream(dev).cuda_stream
        st = self._L.gs_sample(self._ctx, ctypes.byref(b), ctypes.byref(o), ctypes.c_void_p(stream))
        del keep
        if st != _lib.GS_OK:
            _raise(st, self._ctx)
        return out

    def bind(self, logits, params, *, softcap: float = 0.0, history=None, history_len=None, mask_table=None,
             mask_state=None, rng_state=None, uniforms=None, logprob: bool = False, candidates: int = 0,
             stream=None, history_count=None) -> "BoundSample":
        """A reusable ``sample`` call for a decode loop: every argument but the logits is
        fixed (the params, the history, mask and state tensors are read afresh on the
        device at each call, so their contents may change; their storage may not).  Each
        call takes logits of ``logits``' shape, dtype and row stride and returns the same
        output tensors, rewritten."""
        return BoundSample(self, logits, params, softcap=softcap, history=history, history_len=history_len,
                           mask_table=mask_table, mask_state=mask_state, rng_state=rng_state, uniforms=uniforms,
                           logprob=logprob, candidates=candidates, stream=stream, history_count=history_count)

    # ---------------------------------------------------------------- vocabulary shards
    def shard_record_bytes(self, params, vocab_total: int, history_stride: int = 0) -> int:
        """Bytes of one row's shard record (gs_shard_record_bytes)."""
        parr = _params_array(params)
        n = self._L.gs_shard_record_bytes(parr, len(parr), int(vocab_total), int(history_stride))
        if n < 0:
            raise ValueError("invalid shard record geometry")
        return int(n)

    def shard_partials(self, logits, params, *, vocab_offset: int, vocab_total: int, softcap: float = 0.0,
                       history=None, history_len=None, mask_table=None, mask_state=None, logprob: bool = False,
                       records=None, stream=None):
        """Streams this GPU's vocabulary shard ``logits`` [rows, shard_vocab] (global ids
        [vocab_offset, vocab_offset + shard_vocab)) and returns its per-row records, a uint8
        device tensor [rows, record_bytes] (gs_shard_partials).  History ids are global and
        ``mask_table`` covers the whole vocabulary; ``logprob`` records the raw sums a merge
        with log-probabilities needs."""
        import torch
        b, keep = self.make_batch(logits, params, softcap=softcap, history=history, history_len=history_len,
                                  mask_table=mask_table, mask_state=mask_state)
        hstride = b.history_stride if history is not None else 0
        nbytes = self.shard_record_bytes(params, vocab_total, hstride)
        rows = logits.shape[0]
        if records is None:
            records = torch.empty((rows, nbytes), dtype=torch.uint8, device=logits.device)
        if records.numel() < rows * nbytes:
            raise ValueError("records buffer too small")
        if stream is None:
            stream = torch.cuda.current_stream(logits.device).cuda_stream
        st = self._L.gs_shard_partials(self._ctx, ctypes.byref(b), int(vocab_offset), int(vocab_total),
                                       1 if logprob else 0, ctypes.c_void_p(records.data_ptr()),
                                       ctypes.c_void_p(stream))
        del keep
        if st != _lib.GS_OK:
            _raise(st, self._ctx)
        return records

    def shard_merge(self, gathered, params, *, rows: int, shards: int, vocab_total: int, history_stride: int = 0,
                    mask_table=None, mask_state=None, rng_state=None, uniforms=None, logprob: bool = False,
                    candidates: int = 0, stream=None) -> SampleResult:
        """Merges the all-gathered shard records ([shards][rows] records, uint8 device
        tensor) and samples the rows exactly as ``sample`` would on whole rows
        (gs_shard_merge).  Every rank passing the same records gets the same result."""
        import torch
        dev = gathered.device
        parr = _params_array(params)
        b = GsBatch()
        b.dtype = _lib.GS_DTYPE_F32
        b.rows = rows
        b.vocab = int(vocab_total)
        b.row_stride = int(vocab_total)
        b.params_count = len(parr)
        b.params = ctypes.cast(parr, ctypes.c_void_p)
        hist_dummy = None
        if history_stride > 0:
            hist_dummy = torch.zeros(1, dtype=torch.int32, device=dev)  # record layout only
            b.history = hist_dummy.data_ptr()
            b.history_len = hist_dummy.data_ptr()
            b.history_stride = int(history_stride)
        if mask_table is not None:
            b.mask_table = mask_table.data_ptr()
            b.mask_states = mask_table.shape[0]
            b.mask_words = mask_table.stride(0) if mask_table.shape[0] > 1 else mask_table.shape[1]
            b.mask_state = mask_state.data_ptr()
        if rng_state is not None:
            b.rng_state = rng_state.data_ptr()
        if uniforms is not None:
            b.uniforms = uniforms.data_ptr()
        out = SampleResult(
            ids=torch.empty(rows, dtype=torch.int32, device=dev),
            flags=torch.empty(rows, dtype=torch.int32, device=dev),
            logprob=torch.empty(rows, dtype=torch.float64, device=dev) if logprob else None,
            cand_ids=torch.empty((rows, candidates), dtype=torch.int32, device=dev) if candidates else None,
            cand_probs=torch.empty((rows, candidates), dtype=torch.float64, device=dev) if candidates else None,
            cand_count=torch.empty(rows, dtype=torch.int32, device=dev) if candidates else None,
        )
        o = GsOutputs()
        o.ids = _ptr(out.ids)
        o.flags = _ptr(out.flags)
        o.logprob = _ptr(out.logprob)
        o.cand_ids = _ptr(out.cand_ids)
        o.cand_probs = _ptr(out.cand_probs)
        o.cand_count = _ptr(out.cand_count)
        o.cand_cap = candidates
        if stream is None:
            stream = torch.cuda.current_stream(dev).cuda_stream
        st = self._L.gs_shard_merge(self._ctx, ctypes.byref(b), int(shards), ctypes.c_void_p(gathered.data_ptr()),
                                    ctypes.byref(o), ctypes.c_void_p(stream))
        del hist_dummy
        if st != _lib.GS_OK:
            _raise(st, self._ctx)
        return out

    def sample_host(self, logits: np.ndarray, params, *, softcap: float = 0.0, history: np.ndarray | None = None,
                    history_len: np.ndarray | None = None, mask_table=None, mask_state: np.ndarray | None = None,
                    rng_state: np.ndarray | None = None, uniforms: np.ndarray | None = None, logprob: bool = False,
                    candidates: int = 0, stream: int = 0, dtype: int = _lib.GS_DTYPE_F32,
                    history_count: np.ndarray | None = None):
        """gs_sample_host: every buffer in host memory (numpy) except ``mask_table`` (a device tensor:
        compiled constraint tables stay resident).  Synchronous; raises the reference's error for
        the first failing row.  ``rng_state`` (float64) is advanced in place."""
        if logits.ndim != 2:
            raise ValueError("logits must be [rows, vocab]")
        rows, vocab = logits.shape
        parr = _params_array(params)
        b = GsBatch()
        b.logits = logits.ctypes.data
        b.dtype = dtype
        b.rows = rows
        b.vocab = vocab if dtype == _lib.GS_DTYPE_F32 else vocab
        b.row_stride = logits.strides[0] // logits.itemsize
        b.softcap = float(softcap)
        b.params_count = len(parr)
        b.params = ctypes.cast(parr, ctypes.c_void_p)
        if history is not None:
            b.history = history.ctypes.data
            b.history_len = history_len.ctypes.data
            b.history_stride = history.strides[0] // 4
            if history_count is not None:
                if history_count.dtype != np.int32 or history_count.shape != history.shape or \
                        history_count.strides != history.strides:
                    raise ValueError("history_count must be int32 with the history's shape and strides")
                b.history_count = history_count.ctypes.data
        if mask_table is not None:
            b.mask_table = mask_table.data_ptr()
            b.mask_states = mask_table.shape[0]
            b.mask_words = mask_table.stride(0)
            b.mask_state = mask_state.ctypes.data
        if rng_state is not None:
            b.rng_state = rng_state.ctypes.data
        if uniforms is not None:
            b.uniforms = uniforms.ctypes.data
        ids = np.empty(rows, dtype=np.int32)
        flags = np.empty(rows, dtype=np.uint32)
        lp = np.empty(rows, dtype=np.float64) if logprob else None
        cid = np.empty((rows, candidates), dtype=np.int32) if candidates else None
        cpr = np.empty((rows, candidates), dtype=np.float64) if candidates else None
        cc = np.empty(rows, dtype=np.int32) if candidates else None
        o = GsOutputs()
        o.ids = ids.ctypes.data
        o.flags = flags.ctypes.data
        o.logprob = lp.ctypes.data if lp is not None else None
        o.cand_ids = cid.ctypes.data if cid is not None else None
        o.cand_probs = cpr.ctypes.data if cpr is not None else None
        o.cand_count = cc.ctypes.data if cc is not None else None
        o.cand_cap = candidates
        st = self._L.gs_sample_host(self._ctx, ctypes.byref(b), ctypes.byref(o), ctypes.c_void_p(stream))
        if st != _lib.GS_OK:
            _raise(st, self._ctx)
        return SampleResult(ids=ids, flags=flags, logprob=lp, cand_ids=cid, cand_probs=cpr, cand_count=cc)


_samplers: dict[int, GpuSampler] = {}


def default_sampler(device: int = 0) -> GpuSampler:
    s = _samplers.get(device)
    if s is None:
        s = GpuSampler(device)
        _samplers[device] = s
    return s


# ------------------------------------------------------------------- reference mirror


def sample_token(raw_logits, history: Sequence[int], config: dict, random: SeededRandom | Callable[[], float],
                 *, softcap: float = 0.0, sampler: GpuSampler | None = None) -> int:
    """sampleToken (src/runtime/sampling.ts:18-65) on the GPU.

    ``raw_logits``: a CUDA tensor [V] (float32/bfloat16) or a host sequence of numbers
    (then the logits are uploaded, as the reference's readback boundary would be crossed
    the other way).  ``random``: a SeededRandom (its state is advanced on the device) or
    any callable returning a number in [0, 1), called exactly once when temperature != 0,
    as the reference does.
    """
    import torch
    n = raw_logits.numel() if isinstance(raw_logits, torch.Tensor) else len(raw_logits)
    if n == 0:
        raise ValueError("Cannot sample empty logits")
    recent = windowed_history(history, int(config["repetitionWindow"]))
    counts = None
    if len(recent) > _lib.MAX_HISTORY:  # a long window: its distinct ids with their counts
        recent, counts = compact_history(recent)
        if len(recent) > _lib.MAX_HISTORY:
            raise SamplerError(_lib.GS_EUNSUPPORTED,
                               f"repetition window holds more than {_lib.MAX_HISTORY} distinct ids")
    params = params_from_config(config)
    use_state = isinstance(random, SeededRandom)
    uniform = None
    if not use_state and config["temperature"] != 0:
        uniform = float(random())
    if isinstance(raw_logits, torch.Tensor) and raw_logits.is_cuda:
        s = sampler or default_sampler(raw_logits.device.index or 0)
        dev = raw_logits.device
        logits = raw_logits.reshape(1, -1)
        hist = torch.tensor([recent if recent else [0]], dtype=torch.int32, device=dev)
        hlen = torch.tensor([len(recent)], dtype=torch.int32, device=dev)
        hcnt = None if counts is None else torch.tensor([counts], dtype=torch.int32, device=dev)
        rng = torch.tensor([random.state if use_state else 0.0], dtype=torch.float64, device=dev)
        uni = torch.tensor([uniform if uniform is not None else 0.0], dtype=torch.float64, device=dev)
        res = s.sample(logits, params, softcap=softcap, history=hist, history_len=hlen,
                       rng_state=rng if use_state else None, uniforms=None if use_state else uni,
                       history_count=hcnt)
        flags = int(res.flags.cpu().item())
        tok = int(res.ids.cpu().item())
        _raise_row_flags(flags)
        if use_state:
            random.state = float(rng.cpu().item())
        return tok
    s = sampler or default_sampler(0)
    x = np.ascontiguousarray(np.asarray(raw_logits, dtype=np.float32).reshape(1, -1))
    hist = np.asarray([recent if recent else [0]], dtype=np.int32)
    hlen = np.asarray([len(recent)], dtype=np.int32)
    hcnt = None if counts is None else np.asarray([counts], dtype=np.int32)
    rng = np.asarray([random.state if use_state else 0.0], dtype=np.float64)
    uni = np.asarray([uniform if uniform is not None else 0.0], dtype=np.float64)
    res = s.sample_host(x, params, softcap=softcap, history=hist, history_len=hlen,
                        rng_state=rng if use_state else None, uniforms=None if use_state else uni,
                        history_count=hcnt)
    if use_state:
        random.state = float(rng[0])
    return int(res.ids[0])


class BoundSample:
    """``GpuSampler.bind``: the gs_batch / gs_outputs of a call built once; a call sets the
    logits pointer and runs gs_sample (about 2 us of host time instead of ~12)."""

    def __init__(self, sampler, logits, params, *, softcap, history, history_len, mask_table, mask_state, rng_state,
                 uniforms, logprob, candidates, stream, history_count=None):
        import torch
        self._sampler = sampler
        self._b, self._keep = sampler.make_batch(logits, params, softcap=softcap, history=history,
                                                 history_len=history_len, mask_table=mask_table,
                                                 mask_state=mask_state, rng_state=rng_state, uniforms=uniforms,
                                                 history_count=history_count)
        self._args = (history, history_len, mask_table, mask_state, rng_state, uniforms, history_count)  # (kept alive)
        self.out, self._o = sampler.make_outputs(logits.shape[0], logits.device, logprob, candidates)
        if stream is None:
            stream = torch.cuda.current_stream(logits.device).cuda_stream
        self._shape = (tuple(logits.shape), logits.dtype, logits.stride(0) if logits.shape[0] > 1 else logits.shape[1])
        self._call = sampler._L.gs_sample
        self._refs = (sampler._ctx, ctypes.byref(self._b), ctypes.byref(self._o), ctypes.c_void_p(stream))

    def __call__(self, logits):
        if (tuple(logits.shape), logits.dtype, logits.stride(0) if logits.shape[0] > 1 else logits.shape[1]) != self._shape:
            raise ValueError("bound call: logits of another shape, dtype or row stride")
        self._b.logits = logits.data_ptr()
        st = self._call(*self._refs)
        if st != _lib.GS_OK:
            _raise(st, self._sampler._ctx)
        return self.out


def _raise_row_flags(flags: int):
    if flags & _lib.FLAG_ERR_DEADEND:
        raise SamplerError(_lib.GS_EDEADEND, "Generation constraint reached a tokenization dead end")
    if flags & _lib.FLAG_ERR_NONFINITE:
        raise SamplerError(_lib.GS_ENONFINITE, "logits contain NaN or +Infinity")
    if flags & _lib.FLAG_ERR_INVALID:
        raise ValueError("mask state out of range")
    if flags & _lib.FLAG_ERR_UNSUPPORTED:
        raise SamplerError(_lib.GS_EUNSUPPORTED, "request outside the implemented envelope")
    if flags & _lib.FLAG_ERR_TIMEOUT:
        raise SamplerError(_lib.GS_ETIMEOUT, "device wait timed out")


def token_log_probability(raw_logits, token, *, softcap: float = 0.0, sampler: GpuSampler | None = None) -> float:
    """tokenLogProbability (src/runtime/sampling.ts:67-80) on the GPU."""
    import torch
    n = raw_logits.numel() if isinstance(raw_logits, torch.Tensor) else len(raw_logits)
    if not (isinstance(token, (int, np.integer)) or (isinstance(token, float) and token.is_integer())) \
            or token < 0 or token >= n:
        raise ValueError(f"Token {token} is outside logits length {n}")
    if isinstance(raw_logits, torch.Tensor) and raw_logits.is_cuda:
        x = raw_logits.reshape(1, -1)
        dev_index = raw_logits.device.index or 0
    else:
        x = torch.tensor(np.asarray(raw_logits, dtype=np.float32).reshape(1, -1), device="cuda")
        dev_index = x.device.index or 0
    s = sampler or default_sampler(dev_index)
    dtype = _lib.GS_DTYPE_F32 if x.dtype == torch.float32 else _lib.GS_DTYPE_BF16
    tok = np.asarray([int(token)], dtype=np.int32)
    out = np.empty(1, dtype=np.float64)
    st = s._L.gs_token_log_probability(s.handle, x.data_ptr(), dtype, 1, n, n, float(softcap), tok.ctypes.data,
                                       out.ctypes.data, ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    if st != _lib.GS_OK:
        _raise(st, s.handle)
    return float(out[0])


def mask_constraint_logits(raw_logits, legal_token_ids: Sequence[int], termination_token_ids: Sequence[int],
                           *, sampler: GpuSampler | None = None):
    """maskConstraintLogits (src/runtime/constraints.ts:159-173) on the GPU: a new float32
    tensor, -inf except at legal and termination ids."""
    import torch
    if isinstance(raw_logits, torch.Tensor) and raw_logits.is_cuda:
        x = raw_logits.reshape(-1).to(torch.float32).contiguous()
    else:
        x = torch.tensor(np.asarray(raw_logits, dtype=np.float32).reshape(-1), device="cuda")
    s = sampler or default_sampler(x.device.index or 0)
    legal = torch.tensor(list(legal_token_ids) or [0], dtype=torch.int32, device=x.device)
    term = torch.tensor(list(termination_token_ids) or [0], dtype=torch.int32, device=x.device)
    out = torch.empty_like(x)
    st = s._L.gs_mask_constraint_logits(s.handle, x.data_ptr(), x.numel(), legal.data_ptr(), len(legal_token_ids),
                                        term.data_ptr(), len(termination_token_ids), out.data_ptr(),
                                        ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    if st != _lib.GS_OK:
        _raise(st, s.handle)
    return out


def build_mask_row(vocab: int, legal_token_ids: Sequence[int], termination_token_ids: Sequence[int],
                   *, device: int = 0, sampler: GpuSampler | None = None):
    """One allowed-token bitmask row (int32 words) from the id lists selectConstrainedToken
    hands to maskConstraintLogits (src/runtime/gemma-session.ts:1315-1327)."""
    import torch
    s = sampler or default_sampler(device)
    dev = torch.device("cuda", device)
    legal = torch.tensor(list(legal_token_ids) or [0], dtype=torch.int32, device=dev)
    term = torch.tensor(list(termination_token_ids) or [0], dtype=torch.int32, device=dev)
    row = torch.empty((vocab + 31) // 32, dtype=torch.int32, device=dev)
    st = s._L.gs_build_mask_row(s.handle, vocab, legal.data_ptr(), len(legal_token_ids), term.data_ptr(),
                                len(termination_token_ids), row.data_ptr(),
                                ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    if st != _lib.GS_OK:
        _raise(st, s.handle)
    return row


# src/runtime/gemma-tokenizer.ts:19 and src/runtime/gemma-session.ts:124-125
GEMMA_END_CHANNEL_TOKEN_ID = 101
GEMMA_REQUIRED_REASONING_TOKENS = 16
GEMMA_MAX_REQUIRED_REASONING_TOKENS = 64


def reasoning_mask_rows(has_bytes, *, end_channel_id: int = GEMMA_END_CHANNEL_TOKEN_ID, device: int = 0,
                        sampler: GpuSampler | None = None):
    """maskReasoningLogits (src/runtime/gemma-session.ts:1331-1345) as a two-row bitmask
    table (int32 words, [2, ceil(V/32)]): row 0 allows the ids whose tokenBytes is not null
    (``has_bytes[id]`` true), row 1 also ``end_channel_id``.  Built once per vocabulary;
    a required-reasoning step samples with ``reasoning_mask_state(...)`` as its row's mask
    state over this table instead of masking a copy of the logits every token."""
    import numpy as np
    import torch
    s = sampler or default_sampler(device)
    dev = torch.device("cuda", device)
    hb = torch.as_tensor(np.ascontiguousarray(np.asarray(has_bytes, dtype=bool).astype(np.uint8))).to(dev) \
        if not isinstance(has_bytes, torch.Tensor) else has_bytes.to(device=dev, dtype=torch.uint8).contiguous()
    vocab = hb.numel()
    words = (vocab + 31) // 32
    rows = torch.empty((2, words), dtype=torch.int32, device=dev)
    st = s._L.gs_build_reasoning_mask_rows(s.handle, vocab, hb.data_ptr(), int(end_channel_id), rows.data_ptr(),
                                           words, ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    if st != _lib.GS_OK:
        _raise(st, s.handle)
    return rows


def reasoning_mask_state(reasoning_content_tokens: int) -> int:
    """Row of the reasoning table for a required-reasoning step: the end-of-channel id is
    allowed again once GEMMA_REQUIRED_REASONING_TOKENS reasoning tokens were sampled
    (src/runtime/gemma-session.ts:676-687; at GEMMA_MAX_REQUIRED_REASONING_TOKENS the
    caller emits the end-of-channel id without sampling)."""
    return 1 if reasoning_content_tokens >= GEMMA_REQUIRED_REASONING_TOKENS else 0
