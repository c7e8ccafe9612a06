"""Writes tests/golden/reference_spec_cases.json.

Every case below is a known-answer test of the reference's own test suite
(aribornstein/gemma-webgpu-engine), restated as data: the inputs and the asserted
result, with the spec file and line it comes from.  The reference cannot run in this
container (no Node), so these assertions are the pin for the oracle and, through the
C-ABI, for the CUDA path.

Inputs are rounded to float32 because the production path always samples from a
Float32Array read back from the GPU (src/webgpu/decode-model.ts:183-188); none of the
asserted outcomes depends on that rounding (every decision margin is > 1e-3).
"""
import json
import math
import os

DEFAULT = {  # src/runtime/decoding.ts:16-29
    "temperature": 0.8, "topK": 40, "topP": 0.95, "minP": 0, "typicalP": 1,
    "repetitionPenalty": 1.05, "repetitionWindow": 64, "frequencyPenalty": 0,
    "presencePenalty": 0, "maxNewTokens": 256, "seed": 42, "stopTokenIds": [],
}


def cfg(**kw):
    c = dict(DEFAULT)
    c.update(kw)
    return c


L = [math.log(0.6), math.log(0.3), math.log(0.1)]
sample_cases = [
    {"name": "temperature zero performs greedy decoding", "src": "tests/sampling.spec.ts:13-15",
     "logits": [0.2, 4, 1], "history": [], "config": cfg(temperature=0), "uniform": 0.5, "expect": 1},
    {"name": "top-k one is deterministic", "src": "tests/sampling.spec.ts:17-19",
     "logits": [0.2, 4, 1], "history": [], "config": cfg(topK=1), "uniform": 0.99, "expect": 1},
    {"name": "repetition penalty can move selection away from history", "src": "tests/sampling.spec.ts:30-32",
     "logits": [2, 1.5], "history": [0], "config": cfg(temperature=0, repetitionPenalty=2), "uniform": 0,
     "expect": 1},
    {"name": "zero repetition window disables history penalties", "src": "tests/sampling.spec.ts:34-46",
     "logits": [2, 1.5], "history": [0], "config": cfg(temperature=0, repetitionPenalty=2, repetitionWindow=0),
     "uniform": 0, "expect": 0},
    {"name": "presence and frequency penalties use counts inside the repetition window (a)",
     "src": "tests/sampling.spec.ts:86-95",
     "logits": [2, 1.5], "history": [0, 0],
     "config": cfg(temperature=0, repetitionPenalty=1, repetitionWindow=2, presencePenalty=0.1,
                   frequencyPenalty=0.3), "uniform": 0, "expect": 1},
    {"name": "presence and frequency penalties use counts inside the repetition window (b)",
     "src": "tests/sampling.spec.ts:97-102",
     "logits": [2, 2.1], "history": [0, 1],
     "config": cfg(temperature=0, repetitionPenalty=1, repetitionWindow=1, presencePenalty=0.5,
                   frequencyPenalty=0), "uniform": 0, "expect": 0},
    {"name": "min-p filters tokens relative to the leading probability", "src": "tests/sampling.spec.ts:105-115",
     "logits": L, "history": [], "config": cfg(temperature=1, topK=0, topP=1, typicalP=1, minP=0.6),
     "uniform": 0.99, "expect": 0},
    {"name": "top-p keeps the smallest leading probability mass", "src": "tests/sampling.spec.ts:117-127",
     "logits": L, "history": [], "config": cfg(temperature=1, topK=0, topP=0.5, minP=0, typicalP=1),
     "uniform": 0.99, "expect": 0},
    {"name": "typical-p can select a non-leading token closest to entropy", "src": "tests/sampling.spec.ts:129-139",
     "logits": [math.log(0.45), math.log(0.4), math.log(0.15)], "history": [],
     "config": cfg(temperature=1, topK=0, topP=1, minP=0, typicalP=0.3), "uniform": 0.5, "expect": 1},
]

reproducible = {  # tests/sampling.spec.ts:21-28 (two streams compared with each other)
    "name": "seeded sampling is reproducible", "src": "tests/sampling.spec.ts:21-28",
    "logits": [1, 1, 1], "history": [], "config": cfg(topK=0, topP=1), "seed": 71, "draws": 20,
}

log_probability = {  # tests/sampling.spec.ts:141-146 (toBeCloseTo: 2 decimal digits)
    "src": "tests/sampling.spec.ts:141-146", "logits": L,
    "cases": [{"token": 0, "expect": math.log(0.6)}, {"token": 2, "expect": math.log(0.1)}],
    "error_token": 3, "error_match": "outside logits length",
}

mask = {  # tests/constraints.spec.ts:158-161
    "src": "tests/constraints.spec.ts:158-161", "logits": [1, 2, 3, 4], "legal": [1, 3],
    "termination": [0], "expect": [1, 2, "-inf", 4],
}

validation = {  # tests/sampling.spec.ts:48-64
    "src": "tests/sampling.spec.ts:48-64",
    "input": {"topP": "NaN", "repetitionWindow": -1, "frequencyPenalty": "Infinity", "presencePenalty": -0.1,
              "stopTokenIds": [1, -2]},
    "errors": [
        "topP must be between 0 and 1",
        "repetitionWindow must be a non-negative integer",
        "frequencyPenalty must be finite and non-negative",
        "presencePenalty must be finite and non-negative",
        "stopTokenIds must contain non-negative integers",
    ],
}

generation = {  # tests/sampling.spec.ts:66-84
    "defaults_src": "tests/sampling.spec.ts:66-72",
    "defaults": {"maxNewTokens": 256, "temperature": 0, "repetitionPenalty": 1, "usesGpuGreedy": True},
    "routing_src": "tests/sampling.spec.ts:74-78",
    "routing": [{"temperature": 0.8}, {"repetitionPenalty": 1.1}, {"presencePenalty": 0.1}],
    "stop_src": "tests/sampling.spec.ts:80-84",
    "stop_input": {"stopTokenIds": [262144]}, "stop_error": "Gemma stop token IDs must be below 262144",
}

out = {
    "about": "Known-answer tests of the reference's tests/sampling.spec.ts and tests/constraints.spec.ts, "
             "restated as data by tests/golden/make_reference_spec_cases.py.",
    "default_decoding_config": DEFAULT,
    "sample_cases": sample_cases,
    "reproducible": reproducible,
    "log_probability": log_probability,
    "mask": mask,
    "validation": validation,
    "generation": generation,
}

if __name__ == "__main__":
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_spec_cases.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)
