"""Python handles on the engine's sm_100a kernels.

Each function takes CUDA torch tensors, checks shapes and layouts, and calls the raw launcher of
the native extension on the current stream. The launchers fail loudly: a missing extension on a
GPU host raises, so no test or benchmark silently runs a PyTorch fallback.
"""

from .native import native, scratch  # noqa: F401
from .kernels import (  # noqa: F401
    EPI_BF16,
    EPI_F32,
    EPI_SWIGLU,
    MODE_AUTO,
    MODE_ROWS,
    MODE_SWAP,
    W_BF16,
    W_FP8_BLOCK,
    W_NVFP4,
    W_NVFP4_A4,
    W_FP8_W8A16,
    QuantizedWeight,
    argmax,
    embedding,
    gemm,
    qk_norm_rope_cache,
    rmsnorm,
    paged_decode,
    paged_prefill,
    prefill_work,
    quantize_fp8_block,
    quantize_fp8_rows,
    quantize_nvfp4,
    quantize_nvfp4_input,
    quantize_fp8_input,
    nvfp4_w4a4,
    moe_route,
    moe_align,
    moe_capacity,
    moe_gather,
    moe_combine,
    grouped_gemm,
)
