"""Decoding option surface, kept identical to the reference's.

Mirrors (aribornstein/gemma-webgpu-engine):
  src/runtime/decoding.ts:1-59           DecodingConfig, DEFAULT_DECODING_CONFIG, validateDecodingConfig
  src/runtime/generation-config.ts:47-77 DEFAULT_GENERATION_CONFIG, resolveGemmaGenerationConfig,
                                         usesGemmaGpuGreedy
Error strings and their order are the reference's, so callers see the same messages.
"""
from __future__ import annotations

import math
from typing import Any

VOCAB_SIZE = 262144  # src/runtime/generation-config.ts:10

DEFAULT_DECODING_CONFIG: dict[str, Any] = {  # src/runtime/decoding.ts:16-29
    "temperature": 0.8,
    "topK": 40,
    "topP": 0.95,
    "minP": 0,
    "typicalP": 1,
    "repetitionPenalty": 1.05,
    "repetitionWindow": 64,
    "frequencyPenalty": 0,
    "presencePenalty": 0,
    "maxNewTokens": 256,
    "seed": 42,
    "stopTokenIds": [],
}

DEFAULT_GENERATION_CONFIG: dict[str, Any] = {  # src/runtime/generation-config.ts:47-60
    **DEFAULT_DECODING_CONFIG,
    "temperature": 0,
    "topK": 0,
    "topP": 1,
    "minP": 0,
    "typicalP": 1,
    "repetitionPenalty": 1,
    "repetitionWindow": 0,
    "frequencyPenalty": 0,
    "presencePenalty": 0,
    "maxNewTokens": 256,
    "stopTokenIds": [],
}


def _is_number(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def _finite(v) -> bool:
    return _is_number(v) and math.isfinite(v)


def _is_integer(v) -> bool:
    # Number.isInteger: finite and no fractional part
    return _finite(v) and float(v) == math.floor(float(v))


def validate_decoding_config(input_config: dict) -> dict:
    """validateDecodingConfig (src/runtime/decoding.ts:31-59): {"ok": bool, "errors": [...]}"""
    value = {**DEFAULT_DECODING_CONFIG, **input_config}
    errors: list[str] = []
    t = value["temperature"]
    if not _finite(t) or t < 0:
        errors.append("temperature must be >= 0")
    k = value["topK"]
    if not _is_integer(k) or k < 0:
        errors.append("topK must be a non-negative integer")
    for key in ("topP", "minP", "typicalP"):
        v = value[key]
        if not _finite(v) or v < 0 or v > 1:
            errors.append(f"{key} must be between 0 and 1")
    rp = value["repetitionPenalty"]
    if not _finite(rp) or rp <= 0:
        errors.append("repetitionPenalty must be > 0")
    w = value["repetitionWindow"]
    if not _is_integer(w) or w < 0:
        errors.append("repetitionWindow must be a non-negative integer")
    fp = value["frequencyPenalty"]
    if not _finite(fp) or fp < 0:
        errors.append("frequencyPenalty must be finite and non-negative")
    pp = value["presencePenalty"]
    if not _finite(pp) or pp < 0:
        errors.append("presencePenalty must be finite and non-negative")
    m = value["maxNewTokens"]
    if not _is_integer(m) or m < 1:
        errors.append("maxNewTokens must be a positive integer")
    if not _is_integer(value["seed"]):
        errors.append("seed must be an integer")
    stops = value["stopTokenIds"]
    if not isinstance(stops, (list, tuple)) or any((not _is_integer(s)) or s < 0 for s in stops):
        errors.append("stopTokenIds must contain non-negative integers")
    return {"ok": len(errors) == 0, "errors": errors}


def resolve_gemma_generation_config(options: dict) -> dict:
    """resolveGemmaGenerationConfig (src/runtime/generation-config.ts:62-70)."""
    decoding_keys = set(DEFAULT_GENERATION_CONFIG)
    config = {**DEFAULT_GENERATION_CONFIG, **{k: v for k, v in options.items() if k in decoding_keys}}
    result = validate_decoding_config(config)
    if not result["ok"]:
        raise ValueError(f"Invalid Gemma decoding config: {'; '.join(result['errors'])}")
    if any(s >= VOCAB_SIZE for s in config["stopTokenIds"]):
        raise ValueError(f"Gemma stop token IDs must be below {VOCAB_SIZE}")
    return {**config, "stopTokenIds": list(config["stopTokenIds"])}


def uses_gemma_gpu_greedy(config: dict) -> bool:
    """usesGemmaGpuGreedy (src/runtime/generation-config.ts:72-77)."""
    return (config["temperature"] == 0 and config["repetitionPenalty"] == 1
            and config["frequencyPenalty"] == 0 and config["presencePenalty"] == 0)
