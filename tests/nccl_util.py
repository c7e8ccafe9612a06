"""Builds the fake NCCL library (tests/fake_nccl.c) for the exchange tests."""
import os
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def build_fake_nccl() -> str:
    out = os.path.join(tempfile.mkdtemp(prefix="fake_nccl_"), "libfake_nccl.so")
    subprocess.run(["gcc", "-O1", "-shared", "-fPIC", "-o", out, os.path.join(HERE, "fake_nccl.c"), "-ldl"], check=True)
    return out


def run_worker(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run(["python", os.path.join(HERE, "nccl_worker.py")] + list(args), env=env, capture_output=True,
                          text=True, timeout=timeout)
