"""Spectral norm cache: per-tile |K_high|_F computed once, read by the O(1) decode gate.

Drop-in for ``orthocache_gpu.norm_cache`` (j-arndt/orthocache-gpu,
src/orthocache_gpu/norm_cache.py:21-167).  The key cache of a decoding
sequence never changes, so the high-band Walsh energy of each 64-token key
tile can be computed once (at prefill, or when decoding completes a tile)
and the decode gate then reads one float per tile instead of the tile.

The norms are computed by the library's CUDA kernel
(``oc_tile_high_norms``): one launch scores every tile of every head
(the reference calls ``update_prefill`` per tile with a host sync each).
The cache lives on the GPU; there is no CPU path.
"""

from __future__ import annotations

import torch

from . import _lib
from .fwht_fused_prototype import TILE_SIZE


def _check_walsh(walsh_matrix, tile_size: int) -> None:
    if walsh_matrix is not None and tuple(walsh_matrix.shape) != (tile_size, tile_size):
        raise ValueError(f"walsh_matrix must be ({tile_size}, {tile_size}); the kernel applies the "
                         "natural-order Walsh matrix of generate_walsh_matrix itself")
    if tile_size != TILE_SIZE:
        raise NotImplementedError(f"tile_size={tile_size}: the norm kernel implements 64-token tiles")


def tile_high_norms(keys: torch.Tensor, high_start: int = 48, high_end: int = 64,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """|(W K_tile)[high_start:high_end]|_F of every 64-token tile: keys (H, S, hd) -> (H, S // 64) float32.

    W is the natural-order Walsh matrix / 8 along the tile's tokens; norms
    below 1e-38 read as 0 (norm_cache.py:58-88).  ``out`` (H, >= S // 64)
    float32 with a contiguous last dimension receives the norms in place.
    """
    squeeze = keys.ndim == 2
    if squeeze:
        keys = keys[None]
    heads, seq, hd = keys.shape
    assert seq % TILE_SIZE == 0, f"seq_len {seq} not divisible by tile_size {TILE_SIZE}"
    assert 0 <= high_start <= high_end <= TILE_SIZE, "band must lie in [0, 64]"
    dev = _lib.require_cuda(keys)
    if keys.stride(-1) != 1:
        keys = keys.contiguous()
    tiles = seq // TILE_SIZE
    if out is None:
        out = torch.empty((heads, tiles), dtype=torch.float32, device=dev)
    assert out.dtype == torch.float32 and out.stride(-1) == 1 and out.shape[-1] >= tiles
    _lib.check(_lib.load().oc_tile_high_norms(
        keys.data_ptr(), _lib.dtype_code(keys), heads, seq, hd, keys.stride(0), keys.stride(1),
        high_start, high_end, out.data_ptr(), out.stride(0), _lib.stream_ptr(dev)), "tile_high_norms")
    return out[0] if squeeze else out


class SpectralNormCache:
    """Precomputed K-tile high-band norms for the O(1) decode-phase gate (norm_cache.py:21-167).

    ``cache`` (num_kv_heads, max_tiles) float32 and ``valid_tiles``
    (num_kv_heads,) int32 live on ``device`` (a CUDA device).
    """

    def __init__(self, num_kv_heads: int, max_tiles: int, device):
        self.cache = torch.zeros(num_kv_heads, max_tiles, dtype=torch.float32, device=device)
        self.valid_tiles = torch.zeros(num_kv_heads, dtype=torch.int32, device=device)
        self.num_kv_heads = num_kv_heads
        self.max_tiles = max_tiles
        self.device = device
        self._populated = False

    def update_prefill(self, kv_head: int, tile_idx: int, k_tile: torch.Tensor, walsh_matrix: torch.Tensor,
                       high_start: int, high_end: int):
        """Norm of one tile k_tile (64, hd) into cache[kv_head, tile_idx] (norm_cache.py:58-88).

        No host synchronisation (the reference reads the norm back with ``.item()``).
        """
        _check_walsh(walsh_matrix, k_tile.shape[0])
        k = k_tile.to(self.cache.device)
        tile_high_norms(k[None], high_start, high_end, out=self.cache[kv_head:kv_head + 1, tile_idx:])
        self.valid_tiles[kv_head].clamp_(min=tile_idx + 1)
        self._populated = True

    def populate_from_keys(self, keys: torch.Tensor, walsh_matrix: torch.Tensor, tile_size: int = TILE_SIZE,
                           high_start: int = 48, high_end: int = 64):
        """All tiles of keys (num_kv_heads, seq_len, hd) in one launch (norm_cache.py:90-117)."""
        _check_walsh(walsh_matrix, tile_size)
        kvh, seq, _ = keys.shape
        heads = min(kvh, self.num_kv_heads)
        tiles = min(seq // tile_size, self.max_tiles)
        if heads > 0 and tiles > 0:
            tile_high_norms(keys[:heads, : tiles * tile_size], high_start, high_end, out=self.cache[:heads])
            self.valid_tiles[:heads].clamp_(min=tiles)
            self._populated = True
        return self

    def append_tiles(self, keys: torch.Tensor, first_tile: int, high_start: int = 48, high_end: int = 64):
        """Norms of the whole tiles of keys (num_kv_heads, n*64, hd) into tiles [first_tile, first_tile + n).

        Extension for decoding: when the key cache completes a tile, its norm
        is added without touching the others.
        """
        n = keys.shape[1] // TILE_SIZE
        if n:
            assert first_tile + n <= self.max_tiles, "append beyond max_tiles"
            tile_high_norms(keys[:, : n * TILE_SIZE], high_start, high_end,
                            out=self.cache[: keys.shape[0], first_tile:])
            self.valid_tiles[: keys.shape[0]].clamp_(min=first_tile + n)
            self._populated = True
        return self

    def get_norm(self, kv_head: int, tile_idx: int) -> float:
        """Cached |K_high|_F of one tile (synchronising read)."""
        return self.cache[kv_head, tile_idx].item()

    def get_norms_batch(self, kv_head: int) -> torch.Tensor:
        n = self.valid_tiles[kv_head].item()
        return self.cache[kv_head, :n]

    @property
    def is_populated(self) -> bool:
        return self._populated

    @property
    def memory_bytes(self) -> int:
        return self.cache.nelement() * self.cache.element_size()

    def summary(self) -> str:
        total_tiles = self.valid_tiles.sum().item()
        return (f"SpectralNormCache: {self.num_kv_heads} heads × {self.max_tiles} max_tiles, "
                f"{total_tiles} populated, {self.memory_bytes / 1024:.1f} KB")


def create_norm_cache_for_model(model_config, max_seq_len: int = 32768, tile_size: int = TILE_SIZE,
                                device=None) -> SpectralNormCache:
    """A cache sized for a model config with ``num_key_value_heads`` (norm_cache.py:146-167).

    ``device`` defaults to the current CUDA device (the reference defaults to the CPU).
    """
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return SpectralNormCache(model_config.num_key_value_heads, max_seq_len // tile_size, device)
