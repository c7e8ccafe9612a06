"""The Node-API addon (gemma-webgpu-engine_b200/node/gsampler_napi.cc) built here against a
stand-in Node-API header and runtime (tests/napi/): its argument checks on the CPU, and on
the GPU its sampleHost against the package's sample_token on the same logits, window,
config and random() value (both through libgsampler; Node itself is not in this image)."""
from __future__ import annotations

import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "gemma-webgpu-engine_b200")
KEYS = ("temperature", "topP", "minP", "typicalP", "repetitionPenalty", "presencePenalty", "frequencyPenalty", "topK")


@pytest.fixture(scope="module")
def driver(tmp_path_factory, pkg):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    pkg._lib.lib()  # (libgsampler.so is built)
    exe = str(tmp_path_factory.mktemp("napi") / "napi_driver")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I" + os.path.join(ROOT, "tests", "napi"),
                    "-I" + os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "napi", "fake_napi.cc"),
                    os.path.join(PKG_DIR, "node", "gsampler_napi.cc"), "-L" + PKG_DIR, "-lgsampler",
                    "-Wl,-rpath," + PKG_DIR, "-o", exe], check=True)
    return exe


def call(driver, tmp_path, logits, ids, counts, cfg, uniform, softcap=0.0):
    blob = struct.pack("<q", len(logits)) + np.asarray(logits, np.float32).tobytes() + struct.pack("<q", len(ids))
    blob += np.asarray(ids, np.int32).tobytes() + np.asarray(counts, np.int32).tobytes()
    blob += np.asarray([cfg[k] for k in KEYS], np.float64).tobytes() + struct.pack("<dd", uniform, softcap)
    path = tmp_path / "in.bin"
    path.write_bytes(blob)
    out = subprocess.run([driver, str(path)], capture_output=True, text=True, check=True).stdout.strip()
    kind, _, rest = out.partition(" ")
    return int(rest) if kind == "id" else rest


CFG = dict(temperature=0.8, topK=40, topP=0.95, minP=0.0, typicalP=1.0, repetitionPenalty=1.1, presencePenalty=0.5,
           frequencyPenalty=0.3, repetitionWindow=64)


def test_argument_errors_before_any_device_work(driver, tmp_path):
    assert call(driver, tmp_path, [], [], [], CFG, 0.5) == "Cannot sample empty logits"
    many = list(range(5000))
    assert "4096 distinct ids" in call(driver, tmp_path, [1.0, 2.0], many, [1] * len(many), CFG, 0.5)
    for bad in (2.5, -1.0, float("nan"), float("inf")):  # validateDecodingConfig's topK rule
        assert call(driver, tmp_path, [1.0, 2.0], [], [], dict(CFG, topK=bad), 0.5) == \
            "topK must be a non-negative integer", bad


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["topk", "greedy", "long_window", "topk0", "softcap"])
def test_sample_host_matches_sample_token(pkg, driver, tmp_path, case):
    import torch
    g = np.random.default_rng(len(case))
    V = 262144
    x = (g.standard_normal(V) * 2.0).astype(np.float32)
    history = [int(v) for v in g.integers(0, V, 200)] + [int(np.argmax(x))] * 3
    cfg = dict(CFG)
    softcap = 0.0
    if case == "greedy":
        cfg["temperature"] = 0.0
    elif case == "long_window":
        pool = g.integers(0, V, 900)
        history = [int(v) for v in pool[g.integers(0, len(pool), 7000)]]
        cfg["repetitionWindow"] = 6500
    elif case == "topk0":
        cfg.update(topK=0, topP=0.9)
    elif case == "softcap":
        x *= 10.0
        softcap = 30.0
    u = float(g.random())
    recent = pkg.windowed_history(history, cfg["repetitionWindow"])
    ids, counts = pkg.compact_history(recent)
    got = call(driver, tmp_path, x, ids, counts, cfg, u, softcap)
    want = pkg.sample_token(torch.from_numpy(x).cuda(), history, cfg, lambda: u, softcap=softcap)
    assert got == want, (case, got, want)
