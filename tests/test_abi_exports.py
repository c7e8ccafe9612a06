"""The C-ABI library loads on a machine without a GPU and exports every entry point that
include/gsampler.h declares (no compute call is made here)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "gsampler.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gs_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_expected_symbols(pkg):
    syms = header_symbols()
    assert syms == sorted(pkg._lib.EXPORTS)


def test_library_exports_every_header_symbol(pkg):
    lib = pkg._lib.lib()
    for name in header_symbols():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_structs_match_header_layout(pkg, tmp_path):
    """ctypes mirrors of gs_params / gs_batch / gs_outputs have the C compiler's layout."""
    import subprocess
    structs = {"gs_params": pkg._lib.GsParams, "gs_batch": pkg._lib.GsBatch, "gs_outputs": pkg._lib.GsOutputs,
               "gs_dfa_desc": pkg._lib.GsDfaDesc, "gs_vocab_bytes_desc": pkg._lib.GsVocabBytesDesc,
               "gs_lm_head_desc": pkg._lib.GsLmHeadDesc}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "gsampler.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines())
    for cname, cls in structs.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, f"{cname}.{f}"


def test_no_cpu_fallback_without_device(pkg):
    import torch
    if torch.cuda.is_available():
        return
    import pytest
    with pytest.raises(pkg.SamplerError):
        pkg.GpuSampler(0)


def test_lm_head_entry_points_reject_null_handles(pkg):
    # argument checks that run before any CUDA call (no device needed)
    L = pkg._lib.lib()
    assert L.gs_lm_head_fused_calls(None) == -1
    assert L.gs_lm_head_sample(None, None, 0, None, None, None, None) == pkg._lib.GS_EINVAL
    assert L.gs_lm_head_logits(None, None, 0, None, 0, None, 0, None) == pkg._lib.GS_EINVAL
    assert L.gs_lm_head_set_route(None, pkg._lib.LM_ROUTE_FUSED) == pkg._lib.GS_EINVAL


def test_prepare_params_matches_per_config_conversion():
    """prepare_params (the vectorised conversion a decode loop can do once) gives the same
    gs_params bytes as converting each DecodingConfig on its own."""
    import importlib
    S = importlib.import_module("gemma-webgpu-engine_b200.sampling")
    ps = [dict(temperature=0.1 * i, topK=[0, 40, 2**40][i % 3], topP=0.9, minP=0.01 * (i % 5), typicalP=1.0,
               repetitionPenalty=1.0 + 0.1 * i, presencePenalty=0.5, frequencyPenalty=0.25, repetitionWindow=64)
          for i in range(37)]
    a = S.prepare_params(ps)
    b = (S.GsParams * len(ps))(*[S.params_from_config(p) for p in ps])
    assert bytes(a) == bytes(b)
    assert S.prepare_params(a) is a


def test_compact_history_keeps_first_occurrence_order_and_counts(pkg):
    """A window as distinct ids in order of first occurrence with their counts (the form
    gs_batch.history_count takes); out-of-range and negative ids are kept as entries, as
    the reference's Map keeps them (src/runtime/sampling.ts:21-27)."""
    import collections
    rng = __import__("numpy").random.default_rng(3)
    window = [int(v) for v in rng.integers(-3, 50, 5000)]
    ids, counts = pkg.compact_history(window)
    assert len(ids) == len(set(window))
    assert ids == list(dict.fromkeys(window))
    c = collections.Counter(window)
    assert counts == [c[i] for i in ids]
    assert pkg.compact_history([]) == ([], [])


def test_history_count_must_match_the_history(pkg):
    """history_count is read beside history with the same strides: mismatches are refused
    on the host (no device needed)."""
    import pytest
    import torch
    s = object.__new__(pkg.GpuSampler)  # make_batch needs no context
    logits = torch.zeros((2, 64), dtype=torch.float32)
    hist = torch.zeros((2, 8), dtype=torch.int32)
    hlen = torch.full((2,), 8, dtype=torch.int32)
    p = [dict(temperature=1.0, topK=5, topP=1.0, minP=0.0, typicalP=1.0, repetitionPenalty=1.1,
              presencePenalty=0.0, frequencyPenalty=0.0)]
    b, _ = s.make_batch(logits, p, history=hist, history_len=hlen, history_count=torch.ones((2, 8), dtype=torch.int32))
    assert b.history_count != 0
    for bad in (torch.ones((2, 7), dtype=torch.int32), torch.ones((2, 8), dtype=torch.int64)):
        with pytest.raises(ValueError):
            s.make_batch(logits, p, history=hist, history_len=hlen, history_count=bad)
    with pytest.raises(ValueError):
        s.make_batch(logits, p, history_count=torch.ones((2, 8), dtype=torch.int32))
