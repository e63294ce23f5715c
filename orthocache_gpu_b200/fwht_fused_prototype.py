"""Walsh matrix, band constants and the ζ eviction mask on the GPU.

Drop-in for the reference's ``orthocache_gpu.triton_kernels.fwht_fused_prototype``
(j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/fwht_fused_prototype.py).
The scoring runs in the library's sm_100a CUDA kernel (closed-form band
energies of the 64-point natural-order Walsh transform along the token axis
of each tile); there is no Triton and no CPU fallback.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

TILE_SIZE = 64
# 64-point natural-order band boundaries (fwht_fused_prototype.py:42-50)
BAND_DC_64 = 0
BAND_LOW_64 = (1, 8)
BAND_MID_64 = (8, 32)
BAND_HIGH_64 = (32, 64)


def generate_walsh_matrix(n: int) -> torch.Tensor:
    """Natural-order (Sylvester) Hadamard matrix scaled by 1/sqrt(n), float32.

    Same construction as fwht_fused_prototype.py:57-80; used for tests and
    analysis only (the kernels never materialise it).
    """
    assert n > 0 and (n & (n - 1)) == 0, f"n must be a power of 2, got {n}"
    h = torch.ones((1, 1), dtype=torch.float32)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], dim=1), torch.cat([h, -h], dim=1)], dim=0)
    return h / (n ** 0.5)


def _check_tile_size(tile_size: int) -> None:
    assert (tile_size & (tile_size - 1)) == 0 and tile_size > 0, f"tile_size ({tile_size}) must be a power of 2"
    if tile_size != TILE_SIZE:
        raise NotImplementedError(
            f"tile_size={tile_size}: the B200 kernels implement the 64-token tile of the reference's "
            "band definition (BAND_LOW_64 / BAND_HIGH_64)")


def triton_fwht_eviction(
    keys: torch.Tensor,
    zeta_max: float,
    tile_size: int = TILE_SIZE,
    return_zeta: bool = False,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Per-tile ζ = E_high / (E_low + 1e-6) and the retain mask (True = keep).

    Same contract as the reference's ``triton_fwht_eviction``
    (fwht_fused_prototype.py:255-322): keys (num_tiles*tile_size, head_dim);
    mask[t] = ζ_t <= zeta_max (compared in float32, so a NaN ζ is evicted).
    The name is kept for drop-in compatibility; the kernel is CUDA, not Triton.
    """
    assert keys.ndim == 2, f"keys must be 2D (tokens, head_dim), got {keys.shape}"
    num_tokens, head_dim = keys.shape
    num_tiles = num_tokens // tile_size
    assert num_tokens == num_tiles * tile_size, f"seq_len {num_tokens} not divisible by tile_size {tile_size}"
    _check_tile_size(tile_size)
    dev = _lib.require_cuda(keys)
    keys = _lib.prepare_kv(keys)
    mask = torch.empty(num_tiles, dtype=torch.bool, device=dev)
    zeta = torch.empty(num_tiles, dtype=torch.float32, device=dev) if return_zeta else None
    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    _lib.check(_lib.load().oc_fwht_eviction(keys.data_ptr(), _lib.dtype_code(keys), num_tokens, head_dim, keys.stride(0),
                                    float(zeta_max), mask.data_ptr(), _lib.ptr(zeta),
                                    ws.status_ptr, stream), "triton_fwht_eviction")
    return mask, zeta
