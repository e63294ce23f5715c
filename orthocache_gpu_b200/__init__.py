"""orthocache_gpu_b200: B200-native fused spectral-eviction decode attention.

A drop-in for the fused decode path of OrthoCache (j-arndt/orthocache-gpu):
the same public functions, argument meaning, assertion messages and output
dtypes, computed by hand-written sm_100a CUDA kernels behind a C ABI
(``include/orthocache_b200.h``, ``liborthocache_b200.so``).  Importing the
package needs no GPU; every compute call needs CUDA tensors and the built
library and raises otherwise (there is no CPU fallback).
"""

from ._lib import check_status
from .fused_eviction import fused_orthocache_attention, fused_orthocache_attention_v2
from .fwht_fused_prototype import (
    BAND_DC_64,
    BAND_HIGH_64,
    BAND_LOW_64,
    BAND_MID_64,
    TILE_SIZE,
    generate_walsh_matrix,
    triton_fwht_eviction,
)
from .decode_gate import (
    apply_decode_mask,
    apply_decode_mask_vectorized,
    compute_q_high_norm_exact,
    decode_gate,
    fused_orthocache_attention_cached,
)
from .gqa_eviction import fused_orthocache_attention_v3_gqa
from .paged_eviction import fused_orthocache_attention_paged
from .norm_cache import SpectralNormCache, create_norm_cache_for_model, tile_high_norms
from .pipeline import BypassFlag, GPUProfile, TelemetryLevel, format_bypass_reason, orthocache_forward

__version__ = "0.1.0"

__all__ = [
    "fused_orthocache_attention",
    "fused_orthocache_attention_v2",
    "fused_orthocache_attention_v3_gqa",
    "fused_orthocache_attention_paged",
    "triton_fwht_eviction",
    "generate_walsh_matrix",
    "orthocache_forward",
    "TelemetryLevel",
    "BypassFlag",
    "GPUProfile",
    "format_bypass_reason",
    "check_status",
    "decode_gate",
    "compute_q_high_norm_exact",
    "apply_decode_mask",
    "apply_decode_mask_vectorized",
    "fused_orthocache_attention_cached",
    "SpectralNormCache",
    "create_norm_cache_for_model",
    "tile_high_norms",
    "TILE_SIZE",
    "BAND_DC_64",
    "BAND_LOW_64",
    "BAND_MID_64",
    "BAND_HIGH_64",
]
