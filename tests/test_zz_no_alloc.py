"""gs_sample_noalloc, the allocation-free entry point, against gs_sample.

Callers such as a serving runtime whose memory pool already owns the device, or a
real-time decode loop that cannot afford cudaMalloc's device-wide synchronisation, use
gs_sample_noalloc: same kernels, scratch in a fixed device array instead of a context
workspace.  Its outputs must equal gs_sample's bit for bit, call after call (the shared
scratch keeps the previous call's contents, which must not leak into the next result).

This file is collected last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
import ctypes
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _outputs(torch, rows, cap, dev):
    return {
        "ids": torch.full((rows,), -7, dtype=torch.int32, device=dev),
        "flags": torch.zeros(rows, dtype=torch.int32, device=dev),
        "logprob": torch.zeros(rows, dtype=torch.float64, device=dev),
        "cand_ids": torch.zeros((rows, cap), dtype=torch.int32, device=dev),
        "cand_probs": torch.zeros((rows, cap), dtype=torch.float64, device=dev),
        "cand_count": torch.zeros(rows, dtype=torch.int32, device=dev),
    }


def _gs_outputs(L, out, cap):
    o = L.GsOutputs()
    for k in ("ids", "flags", "logprob", "cand_ids", "cand_probs", "cand_count"):
        setattr(o, k, out[k].data_ptr())
    o.cand_cap = cap
    return o


@pytest.mark.parametrize("name,rows,per_row", [("C4", 96, False), ("C5", 8, False), ("C3", 40, True),
                                               ("C2", 8, True)])
def test_noalloc_matches_gs_sample_on_two_calls(pkg, name, rows, per_row):
    import torch
    L = pkg._lib
    lib = L.lib()
    W = importlib.import_module("gemma-webgpu-engine_b200.workloads")
    dev = torch.device("cuda", 0)
    wl = W.make(name, device=dev, rows=rows)
    params = wl.params if per_row or len(wl.params) == 1 else wl.params[:1]
    if per_row and len(params) == 1:
        params = params * rows
    cap = 64
    sampler = pkg.GpuSampler(0)
    stream = torch.cuda.current_stream(dev).cuda_stream

    rng_ref = wl.rng_state(dev)
    ref = sampler.sample(wl.logits, params, softcap=wl.softcap, history=wl.history, history_len=wl.history_len,
                         mask_table=wl.mask_table, mask_state=wl.mask_state, rng_state=rng_ref, logprob=True,
                         candidates=cap)
    torch.cuda.synchronize()
    ref_host = {k: getattr(ref, k).cpu().numpy() for k in ("ids", "flags", "logprob", "cand_ids", "cand_probs",
                                                           "cand_count")}
    assert not (ref_host["flags"].view(np.uint32) & L.FLAG_ERRORS).any()

    for call in range(2):
        rng = wl.rng_state(dev)
        b, keep = sampler.make_batch(wl.logits, params, softcap=wl.softcap, history=wl.history,
                                     history_len=wl.history_len, mask_table=wl.mask_table,
                                     mask_state=wl.mask_state, rng_state=rng)
        out = _outputs(torch, rows, cap, dev)
        o = _gs_outputs(L, out, cap)
        st = lib.gs_sample_noalloc(ctypes.byref(b), ctypes.byref(o), ctypes.c_void_p(stream))
        assert st == L.GS_OK, lib.gs_last_error(None)
        torch.cuda.synchronize()
        del keep
        for k, v in ref_host.items():
            got = out[k].cpu().numpy()
            assert np.array_equal(got, v), f"call {call}: {k} differs"
        assert np.array_equal(rng.cpu().numpy(), rng_ref.cpu().numpy()), f"call {call}: rng states differ"
    sampler.close()


def test_noalloc_rejects_requests_beyond_its_scratch(pkg):
    import torch
    L = pkg._lib
    lib = L.lib()
    dev = torch.device("cuda", 0)
    rows = 4096
    logits = torch.zeros((rows, 8192), dtype=torch.float32, device=dev)
    p = L.GsParams(1.0, 1.0, 0.0, 1.0, 1.0, 0.0, 0.0, 1024, 0)
    parr = (L.GsParams * 1)(p)
    b = L.GsBatch()
    b.logits = logits.data_ptr()
    b.dtype = L.GS_DTYPE_F32
    b.rows = rows
    b.vocab = 8192
    b.row_stride = 8192
    b.params_count = 1
    b.params = ctypes.cast(parr, ctypes.c_void_p)
    uni = torch.zeros(rows, dtype=torch.float64, device=dev)
    b.uniforms = uni.data_ptr()
    ids = torch.zeros(rows, dtype=torch.int32, device=dev)
    o = L.GsOutputs()
    o.ids = ids.data_ptr()
    st = lib.gs_sample_noalloc(ctypes.byref(b), ctypes.byref(o), None)
    assert st == L.GS_EUNSUPPORTED
    msg = lib.gs_last_error(None).decode()
    assert "bytes of scratch" in msg and str(L.NOALLOC_SCRATCH_BYTES) in msg
