"""gs_shard_sample (partials + ncclAllGather + merge through the C ABI) on GPU.

With a fake NCCL library on one GPU: one shard covering the vocabulary gives gs_sample's
ids, candidates and probabilities on two calls; an exchange that never completes ends
with GS_ETIMEOUT after the call's bound and the communicator aborted (the fake never
launches anything, so no GPU work waits); a failing exchange gives GS_ENCCL.  With real
NCCL on two GPUs: C5 split in two shards samples the same ids as whole rows on each GPU."""
import os
import tempfile

import pytest

import nccl_util as NU

pytestmark = pytest.mark.gpu


def test_fake_exchange_one_gpu():
    lib = NU.build_fake_nccl()
    r = NU.run_worker(["fake_gpu"], {"GS_NCCL_LIBRARY": lib})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fake_gpu ok" in r.stdout


def test_real_nccl_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import subprocess
    d = tempfile.mkdtemp(prefix="gs_nccl_")
    idfile = os.path.join(d, "id")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen(["python", os.path.join(NU.HERE, "nccl_worker.py"), "real", str(r), "2", idfile,
                               os.path.join(d, f"out{r}")], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True) for r in range(2)]
    outs = [p.communicate(timeout=240)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    res = [open(os.path.join(d, f"out{r}")).read().split() for r in range(2)]
    assert res[0][0] == "1" and res[1][0] == "1", res
    assert res[0][1:] == res[1][1:]
