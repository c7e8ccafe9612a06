"""B200-native decode-sampling path of the Gemma generation engine.

A drop-in for the reference engine's full-logit sampler (aribornstein/gemma-webgpu-engine,
src/runtime/sampling.ts and the constraint mask of src/runtime/constraints.ts): logits
stay on the GPU, hand-written sm_100a kernels (csrc/) apply the soft cap, penalties,
constraint bitmask, temperature, top-k / min-p / typical-p / top-p and the seeded draw,
and only token ids come back.  The C ABI is include/gsampler.h; this package is its
Python host side.
"""
from . import _lib  # noqa: F401
from .lm_head import GpuLmHead  # noqa: F401
from .decoding import (  # noqa: F401
    DEFAULT_DECODING_CONFIG,
    DEFAULT_GENERATION_CONFIG,
    resolve_gemma_generation_config,
    uses_gemma_gpu_greedy,
    validate_decoding_config,
)
from .sampling import (  # noqa: F401
    GpuSampler,
    SampleResult,
    SamplerError,
    SeededRandom,
    build_mask_row,
    compact_history,
    default_sampler,
    mask_constraint_logits,
    params_from_config,
    prepare_params,
    reasoning_mask_rows,
    reasoning_mask_state,
    sample_token,
    token_log_probability,
    windowed_history,
)
