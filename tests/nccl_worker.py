"""Subprocess side of the NCCL exchange tests (libgsampler resolves NCCL once per process,
so each case that needs a particular NCCL library runs in a process of its own).

    python nccl_worker.py host                       the fake library (GS_NCCL_LIBRARY): set-up
                                                     timeout, set-up error, set-up and destroy
    python nccl_worker.py fake_gpu                   the fake library on cuda:0: gs_shard_sample
                                                     over one shard equals gs_sample; an
                                                     exchange that never completes times out
    python nccl_worker.py real RANK WORLD IDFILE OUT real NCCL, rank RANK of WORLD on cuda:RANK
"""
from __future__ import annotations

import ctypes
import importlib
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
pkg = importlib.import_module("gemma-webgpu-engine_b200")
L = pkg._lib
lib = L.lib()


def err():
    m = lib.gs_nccl_last_error(None)
    return m.decode() if m else ""


def fake():
    return ctypes.CDLL(os.environ["GS_NCCL_LIBRARY"])


def host():
    f = fake()
    idb = (ctypes.c_char * 128)()
    assert lib.gs_nccl_unique_id(idb) == L.GS_OK
    assert bytes(idb) == b"F" * 128
    comm = ctypes.c_void_p()
    os.environ["FAKE_NCCL_MODE"] = "init_hang"
    t0 = time.time()
    st = lib.gs_nccl_create(-1, idb, 2, 0, 300, ctypes.byref(comm))
    dt = time.time() - t0
    assert st == L.GS_ETIMEOUT, st
    assert 0.25 < dt < 5.0, dt
    assert "timeout" in err() and not comm.value
    assert f.fake_nccl_aborts() == 1
    os.environ["FAKE_NCCL_MODE"] = "init_error"
    assert lib.gs_nccl_create(-1, idb, 2, 0, 300, ctypes.byref(comm)) == L.GS_ENCCL
    assert "ncclCommInitRankConfig" in err()
    os.environ["FAKE_NCCL_MODE"] = "ok"
    assert lib.gs_nccl_create(-1, idb, 2, 1, 300, ctypes.byref(comm)) == L.GS_OK and comm.value
    assert lib.gs_nccl_destroy(comm) == L.GS_OK
    assert lib.gs_nccl_create(-1, idb, 2, 2, 300, ctypes.byref(comm)) == L.GS_EINVAL  # rank outside [0, nranks)
    print("host ok")


def _c5(dev):
    W = importlib.import_module("gemma-webgpu-engine_b200.workloads")
    return W.make("C5", device=dev)


def fake_gpu():
    import numpy as np
    import torch
    f = fake()
    dev = torch.device("cuda", 0)
    sampler = pkg.GpuSampler(0)
    wl = _c5(dev)
    params = pkg.prepare_params(wl.params)
    ref = sampler.sample(wl.logits, params, softcap=wl.softcap, rng_state=wl.rng_state(dev), candidates=64)
    idb = (ctypes.c_char * 128)()
    lib.gs_nccl_unique_id(idb)
    comm = ctypes.c_void_p()
    os.environ["FAKE_NCCL_MODE"] = "ok"
    assert lib.gs_nccl_create(0, idb, 1, 0, 2000, ctypes.byref(comm)) == L.GS_OK
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        rng = wl.rng_state(dev)
        b, keep = sampler.make_batch(wl.logits, params, softcap=wl.softcap, rng_state=rng)
        out, o = sampler.make_outputs(wl.rows, dev, False, 64)
        st = lib.gs_shard_sample(sampler.handle, comm, ctypes.byref(b), 0, wl.vocab, ctypes.byref(o), 2000,
                                 ctypes.c_void_p(stream))
        assert st == L.GS_OK, (st, err())
        torch.cuda.synchronize()
        assert out.ids.cpu().tolist() == ref.ids.cpu().tolist(), call
        assert np.array_equal(out.cand_ids.cpu().numpy(), ref.cand_ids.cpu().numpy())
        assert np.allclose(out.cand_probs.cpu().numpy(), ref.cand_probs.cpu().numpy(), rtol=1e-12, atol=0)
        del keep
    # an exchange that never completes: the call gives up after its timeout and aborts
    os.environ["FAKE_NCCL_MODE"] = "gather_hang"
    b, keep = sampler.make_batch(wl.logits, params, softcap=wl.softcap, rng_state=wl.rng_state(dev))
    out, o = sampler.make_outputs(wl.rows, dev, False, 0)
    t0 = time.time()
    st = lib.gs_shard_sample(sampler.handle, comm, ctypes.byref(b), 0, wl.vocab, ctypes.byref(o), 300,
                             ctypes.c_void_p(stream))
    assert st == L.GS_ETIMEOUT, (st, err())
    assert time.time() - t0 < 5.0
    assert f.fake_nccl_aborts() == 1
    st = lib.gs_shard_sample(sampler.handle, comm, ctypes.byref(b), 0, wl.vocab, ctypes.byref(o), 300,
                             ctypes.c_void_p(stream))
    assert st == L.GS_ENCCL and "aborted" in err()
    assert lib.gs_nccl_destroy(comm) == L.GS_OK
    # an exchange that fails: GS_ENCCL with the library's message
    os.environ["FAKE_NCCL_MODE"] = "ok"
    assert lib.gs_nccl_create(0, idb, 1, 0, 2000, ctypes.byref(comm)) == L.GS_OK
    os.environ["FAKE_NCCL_MODE"] = "gather_error"
    st = lib.gs_shard_sample(sampler.handle, comm, ctypes.byref(b), 0, wl.vocab, ctypes.byref(o), 2000,
                             ctypes.c_void_p(stream))
    assert st == L.GS_ENCCL and "fake remote error" in err(), (st, err())
    lib.gs_nccl_destroy(comm)
    torch.cuda.synchronize()
    sampler.close()
    print("fake_gpu ok")


def real(rank, world, idfile, outfile):
    import numpy as np
    import torch
    SH = importlib.import_module("gemma-webgpu-engine_b200.sharding")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    sampler = pkg.GpuSampler(rank)
    idb = (ctypes.c_char * 128)()
    if rank == 0:
        assert lib.gs_nccl_unique_id(idb) == L.GS_OK, err()
        with open(idfile + ".tmp", "wb") as fh:
            fh.write(bytes(idb))
        os.replace(idfile + ".tmp", idfile)
    else:
        t0 = time.time()
        while not os.path.exists(idfile):
            assert time.time() - t0 < 60, "no communicator id"
            time.sleep(0.05)
        with open(idfile, "rb") as fh:
            ctypes.memmove(idb, fh.read(128), 128)
    comm = ctypes.c_void_p()
    st = lib.gs_nccl_create(rank, idb, world, rank, 60000, ctypes.byref(comm))
    assert st == L.GS_OK, (st, err())
    wl = _c5(dev)
    off, size = SH.vocab_shards(wl.vocab, world)[rank]
    local = wl.logits[:, off:off + size].contiguous()
    params = pkg.prepare_params(wl.params)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rng = wl.rng_state(dev)
    b, keep = sampler.make_batch(local, params, softcap=wl.softcap, rng_state=rng)
    out, o = sampler.make_outputs(wl.rows, dev, False, 64)
    st = lib.gs_shard_sample(sampler.handle, comm, ctypes.byref(b), off, wl.vocab, ctypes.byref(o), 30000,
                             ctypes.c_void_p(stream))
    assert st == L.GS_OK, (st, err())
    torch.cuda.synchronize()
    rng_w = wl.rng_state(dev)
    whole = sampler.sample(wl.logits, params, softcap=wl.softcap, rng_state=rng_w, candidates=64)
    torch.cuda.synchronize()
    same = out.ids.cpu().tolist() == whole.ids.cpu().tolist() and \
        np.array_equal(out.cand_ids.cpu().numpy(), whole.cand_ids.cpu().numpy()) and \
        np.array_equal(rng.cpu().numpy(), rng_w.cpu().numpy())
    with open(outfile, "w") as fh:
        fh.write(f"{int(same)} {' '.join(str(v) for v in out.ids.cpu().tolist())}\n")
    assert lib.gs_nccl_destroy(comm) == L.GS_OK
    sampler.close()


if __name__ == "__main__":
    cmd = sys.argv[1]
    if cmd == "host":
        host()
    elif cmd == "fake_gpu":
        fake_gpu()
    else:
        real(int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], sys.argv[5])
