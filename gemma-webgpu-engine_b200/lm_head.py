"""The int2 LM head on the GPU: the logits the sampler consumes.

Mirrors the reference's LM head pass (src/webgpu/decode-lm-head.ts): weights packed as
V rows of hidden/16 u32 words (code j of word w at bits 2j..2j+1 multiplies activation
element 16w + j; weight = (code - 2)·rowScale), the final activations and their sum in,
logit = srq(rowScale·(Σ code·a - 2·sumA), outputScale) out.  The dot product is exact
(int8 tensor-core MMA over the activations' srq codes when input_scale != 0; double
sums when 0), see gs_lm_head_desc in include/gsampler.h.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .sampling import SamplerError


class GpuLmHead:
    """Packed weights resident on the sampler's device (gs_lm_head_create)."""

    def __init__(self, sampler, packed, row_scales, input_scale: float = 0.0, output_scale: float = 0.0,
                 route: str = "auto"):
        self._L = _lib.lib()
        packed = np.ascontiguousarray(packed, np.uint32)
        if packed.ndim != 2:
            raise ValueError("packed weights must be [vocab, hidden/16] uint32")
        scales = np.ascontiguousarray(row_scales, np.float32)
        if scales.shape != (packed.shape[0],):
            raise ValueError("row_scales must be [vocab]")
        self.vocab, self.hidden = packed.shape[0], packed.shape[1] * 16
        self.input_scale, self.output_scale = float(np.float32(input_scale)), float(np.float32(output_scale))
        self.device = sampler.device
        self._sampler = sampler  # (keeps the context alive: the head samples on it)
        d = _lib.GsLmHeadDesc(self.vocab, self.hidden, packed.ctypes.data, scales.ctypes.data, self.input_scale,
                              self.output_scale)
        self._h = ctypes.c_void_p()
        st = self._L.gs_lm_head_create(sampler.handle, ctypes.byref(d), ctypes.byref(self._h))
        if st != _lib.GS_OK:
            msg = (self._L.gs_last_error(sampler.handle) or b"").decode()
            raise ValueError(msg) if st == _lib.GS_EINVAL else SamplerError(st, msg)
        self.set_route(route)

    def set_route(self, route: str):
        """Route of sample(): "auto" (the fused route only where it measured faster than
        logits + gs_sample), "fused" (wherever it applies) or "two-step" (never)."""
        codes = {"auto": _lib.LM_ROUTE_AUTO, "fused": _lib.LM_ROUTE_FUSED, "two-step": _lib.LM_ROUTE_TWO_STEP}
        if route not in codes:
            raise ValueError(f"route must be one of {sorted(codes)}")
        st = self._L.gs_lm_head_set_route(self._h, codes[route])
        if st != _lib.GS_OK:
            raise SamplerError(st, (self._L.gs_lm_head_last_error(self._h) or b"").decode())
        self.route = route

    def close(self):
        if self._h:
            self._L.gs_lm_head_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def logits(self, activation, activation_sum, out=None, stream=None):
        """Logits [rows, vocab] float32 (device tensor) of activation [rows, hidden] float32
        and activation_sum [rows] float32 (device tensors)."""
        import torch
        if activation.dtype != torch.float32 or activation.dim() != 2 or activation.shape[1] != self.hidden:
            raise ValueError(f"activation must be float32 [rows, {self.hidden}]")
        if activation.stride(1) != 1:
            raise ValueError("activation rows must be contiguous")
        rows = activation.shape[0]
        s = activation_sum.to(torch.float32).contiguous()
        if s.numel() != rows:
            raise ValueError("activation_sum must hold one value per row")
        if out is None:
            out = torch.empty((rows, self.vocab), dtype=torch.float32, device=activation.device)
        if stream is None:
            stream = torch.cuda.current_stream(activation.device).cuda_stream
        st = self._L.gs_lm_head_logits(self._h, ctypes.c_void_p(activation.data_ptr()), activation.stride(0),
                                       ctypes.c_void_p(s.data_ptr()), rows, ctypes.c_void_p(out.data_ptr()),
                                       out.stride(0), ctypes.c_void_p(stream))
        if st != _lib.GS_OK:
            msg = (self._L.gs_lm_head_last_error(self._h) or b"").decode()
            raise ValueError(msg) if st == _lib.GS_EINVAL else SamplerError(st, msg)
        return out

    def sample(self, activation, activation_sum, params, *, softcap: float = 0.0, history=None, history_len=None,
               mask_table=None, mask_state=None, rng_state=None, uniforms=None, logprob: bool = False,
               candidates: int = 0, stream=None):
        """Activations -> sampled tokens in one call (gs_lm_head_sample): the logits of
        ``logits`` sampled as GpuSampler.sample would, without returning them."""
        import torch
        rows = activation.shape[0]
        if activation.dtype != torch.float32 or activation.dim() != 2 or activation.shape[1] != self.hidden:
            raise ValueError(f"activation must be float32 [rows, {self.hidden}]")
        if activation.stride(1) != 1:
            raise ValueError("activation rows must be contiguous")
        s = activation_sum.to(torch.float32).contiguous()
        if s.numel() != rows:
            raise ValueError("activation_sum must hold one value per row")
        # the batch without logits (shape only): the head computes them
        shape_only = torch.empty((rows, self.vocab), dtype=torch.float32, device="meta")
        b, keep = self._sampler.make_batch(shape_only, params, softcap=softcap, history=history,
                                           history_len=history_len, mask_table=mask_table, mask_state=mask_state,
                                           rng_state=rng_state, uniforms=uniforms)
        b.logits = None
        out, o = self._sampler.make_outputs(rows, activation.device, logprob, candidates)
        if stream is None:
            stream = torch.cuda.current_stream(activation.device).cuda_stream
        st = self._L.gs_lm_head_sample(self._h, ctypes.c_void_p(activation.data_ptr()), activation.stride(0),
                                       ctypes.c_void_p(s.data_ptr()), ctypes.byref(b), ctypes.byref(o),
                                       ctypes.c_void_p(stream))
        del keep
        if st != _lib.GS_OK:
            msg = (self._L.gs_lm_head_last_error(self._h) or b"").decode()
            raise ValueError(msg) if st == _lib.GS_EINVAL else SamplerError(st, msg)
        return out

    @property
    def fused_calls(self) -> int:
        """sample() calls that took the fused route (logits kept on chip, shard-record merge)."""
        return int(self._L.gs_lm_head_fused_calls(self._h))

    def check(self):
        """Raises SamplerError(GS_ETIMEOUT) when a bounded wait inside the kernel ran out
        since the last check (synchronises)."""
        f = ctypes.c_int32()
        st = self._L.gs_lm_head_check(self._h, ctypes.byref(f))
        if st != _lib.GS_OK:
            raise SamplerError(st, (self._L.gs_lm_head_last_error(self._h) or b"").decode())


def synthetic(vocab: int, hidden: int = 1536, rows: int = 1, seed: int = 61, input_scale: float = 0.02):
    """Seeded synthetic LM-head inputs of the reference's shapes: packed int2 weights
    [vocab, hidden/16], row scales, activations on the srq grid of `input_scale` (int8
    codes ~ N(0, 40) clipped) and their float32 sums."""
    g = np.random.default_rng(seed)
    packed = g.integers(0, 1 << 32, size=(vocab, hidden // 16), dtype=np.uint64).astype(np.uint32)
    scales = g.uniform(0.002, 0.02, size=vocab).astype(np.float32)
    q = np.clip(np.rint(g.normal(0.0, 40.0, size=(rows, hidden))), -128, 127).astype(np.float32)
    s = np.float32(input_scale) if input_scale else np.float32(0.02)
    act = (q * s).astype(np.float32)
    act_sum = act.sum(axis=1, dtype=np.float32)
    return packed, scales, act, act_sum
