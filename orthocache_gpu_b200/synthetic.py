"""Seeded synthetic decode workloads with the reference benchmark's tile mixture.

The reference's hero benchmark builds keys as a shuffle of "semantic" tiles
(low-sequency Walsh content along the token axis) and "noise" tiles
(benchmarks/profile_multihead.py:60-119).  The workloads here use the
mixture named for the configurations of this port:

* smooth tile: ``W[:, :8] @ N(0,1)^{8 x hd} + N(0, 0.05^2)`` where ``W`` is
  the 64-point natural-order Walsh matrix, i.e. the first 8 Walsh basis
  vectors along the 64 tokens of the tile;
* noisy tile: iid ``N(0,1)``;
* each tile is smooth with probability ``p_smooth`` (0.5);
* values and queries iid ``N(0,1)``.

Everything is generated with ``numpy.random.default_rng(seed)`` in float32
and cast to the requested dtype by torch, so the same seed gives the same
tensors on every machine of this image.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

TILE = 64


def walsh(n: int) -> np.ndarray:
    """Natural-order Hadamard matrix / sqrt(n) (float32)."""
    h = np.ones((1, 1), dtype=np.float32)
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return (h / np.float32(np.sqrt(n))).astype(np.float32)


def tile_mixture(rng: np.random.Generator, lead: tuple, num_tiles: int, head_dim: int,
                 p_smooth: float = 0.5) -> tuple[np.ndarray, np.ndarray]:
    """Keys of shape (*lead, num_tiles*64, head_dim) and the smooth-tile flags."""
    n = int(np.prod(lead)) * num_tiles if lead else num_tiles
    smooth = rng.random(n) < p_smooth
    tiles = rng.standard_normal((n, TILE, head_dim), dtype=np.float32)
    ns = int(smooth.sum())
    if ns:
        w8 = walsh(TILE)[:, :8]                                      # (64, 8)
        coef = rng.standard_normal((ns, 8, head_dim), dtype=np.float32)
        noise = rng.standard_normal((ns, TILE, head_dim), dtype=np.float32)
        tiles[smooth] = np.matmul(w8, coef) + np.float32(0.05) * noise
    keys = tiles.reshape(*lead, num_tiles * TILE, head_dim)
    return keys, smooth.reshape(*lead, num_tiles) if lead else smooth


def zero_high_band_queries(q: np.ndarray) -> np.ndarray:
    """Zero the upper half of the head_dim Walsh spectrum of every other head.

    Used for the GQA configuration ("half of the query heads have their
    high-band Walsh coefficients zeroed"): natural-order rows [hd/2, hd) of
    the head_dim-point transform are removed from heads 1, 3, 5, ...
    """
    hd = q.shape[-1]
    w = walsh(hd)
    spec = q @ w.T
    spec[..., 1::2, hd // 2:] = 0.0
    return (spec @ w).astype(np.float32)


@dataclass
class DecodeInputs:
    q: np.ndarray
    keys: np.ndarray
    values: np.ndarray
    smooth: np.ndarray

    def torch(self, dtype=torch.float16, device="cpu"):
        """(q, k, v) as torch tensors of ``dtype`` on ``device``."""
        return tuple(torch.from_numpy(a).to(dtype).to(device) for a in (self.q, self.keys, self.values))


def mha_inputs(num_heads: int, seq_len: int, head_dim: int, seed: int = 0,
               p_smooth: float = 0.5) -> DecodeInputs:
    """V1/V2 inputs: q (H, hd), K/V (H, S, hd)."""
    rng = np.random.default_rng(seed)
    keys, smooth = tile_mixture(rng, (num_heads,), seq_len // TILE, head_dim, p_smooth)
    values = rng.standard_normal(keys.shape, dtype=np.float32)
    q = rng.standard_normal((num_heads, head_dim), dtype=np.float32)
    return DecodeInputs(q, keys, values, smooth)


def gqa_inputs(num_kv_heads: int, group: int, seq_len: int, head_dim: int, seed: int = 0,
               batch: int | None = None, zero_high_half: bool = True,
               p_smooth: float = 0.5) -> DecodeInputs:
    """V3 inputs: q (Hq, hd), K/V (KVH, S, hd), with an optional leading batch."""
    rng = np.random.default_rng(seed)
    lead = (num_kv_heads,) if batch is None else (batch, num_kv_heads)
    keys, smooth = tile_mixture(rng, lead, seq_len // TILE, head_dim, p_smooth)
    values = rng.standard_normal(keys.shape, dtype=np.float32)
    qshape = (num_kv_heads * group, head_dim) if batch is None else (batch, num_kv_heads * group, head_dim)
    q = rng.standard_normal(qshape, dtype=np.float32)
    if zero_high_half:
        q = zero_high_band_queries(q)
    return DecodeInputs(q, keys, values, smooth)


@dataclass
class PagedInputs:
    q: np.ndarray            # (B, Hq, hd)
    k_cache: np.ndarray      # (NB, KVH, bs, hd)
    v_cache: np.ndarray
    block_tables: np.ndarray  # (B, max_blocks) int32
    seq_lens: np.ndarray     # (B,) int32

    def torch(self, dtype=torch.float16, device="cpu"):
        q, k, v = (torch.from_numpy(a).to(dtype).to(device) for a in (self.q, self.k_cache, self.v_cache))
        bt = torch.from_numpy(self.block_tables).to(device)
        sl = torch.from_numpy(self.seq_lens).to(device)
        return q, k, v, bt, sl


def paged_inputs(num_seqs: int, num_kv_heads: int, group: int, head_dim: int,
                 block_size: int, min_len: int, max_len: int, seed: int = 0,
                 extra_blocks: int = 0, p_smooth: float = 0.5) -> PagedInputs:
    """Ragged paged cache: lengths U[min_len, max_len] rounded down to 64.

    Pages of all sequences are scattered over a randomly permuted physical
    pool of ``sum(blocks) + extra_blocks`` pages.
    """
    rng = np.random.default_rng(seed)
    lens = rng.integers(min_len, max_len + 1, size=num_seqs)
    lens = np.maximum(lens - lens % TILE, TILE).astype(np.int32)
    nblk = (lens + block_size - 1) // block_size
    max_blocks = int(nblk.max())
    total = int(nblk.sum()) + extra_blocks
    perm = rng.permutation(total).astype(np.int32)
    k_cache = np.zeros((total, num_kv_heads, block_size, head_dim), np.float32)
    v_cache = np.zeros_like(k_cache)
    tables = np.zeros((num_seqs, max_blocks), np.int32)
    pos = 0
    for s in range(num_seqs):
        keys, _ = tile_mixture(rng, (num_kv_heads,), int(lens[s]) // TILE, head_dim, p_smooth)
        vals = rng.standard_normal(keys.shape, dtype=np.float32)
        for b in range(int(nblk[s])):
            pb = int(perm[pos]); pos += 1
            tables[s, b] = pb
            lo, hi = b * block_size, min((b + 1) * block_size, int(lens[s]))
            k_cache[pb, :, : hi - lo] = keys[:, lo:hi]
            v_cache[pb, :, : hi - lo] = vals[:, lo:hi]
        # unused table entries point at a valid page (the kernel must not read them)
        tables[s, int(nblk[s]):] = tables[s, 0]
    q = rng.standard_normal((num_seqs, num_kv_heads * group, head_dim), dtype=np.float32)
    return PagedInputs(q, k_cache, v_cache, tables, lens)


def mha_inputs_device(num_heads: int, seq_len: int, head_dim: int, seed: int = 0,
                      device="cuda", dtype=torch.float16, p_smooth: float = 0.5):
    """The same tile mixture generated on the device with a seeded torch generator.

    Statistically identical to :func:`mha_inputs` (not the same numbers); used
    where inputs are too large to generate on the host quickly.
    Returns (q, keys, values) of ``dtype``.
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nt = seq_len // TILE
    keys = torch.randn((num_heads * nt, TILE, head_dim), generator=g, device=device)
    smooth = torch.rand(num_heads * nt, generator=g, device=device) < p_smooth
    w8 = torch.from_numpy(walsh(TILE)[:, :8]).to(device)
    coef = torch.randn((num_heads * nt, 8, head_dim), generator=g, device=device)
    sm = torch.matmul(w8, coef) + 0.05 * torch.randn(keys.shape, generator=g, device=device)
    keys = torch.where(smooth[:, None, None], sm, keys).reshape(num_heads, seq_len, head_dim)
    values = torch.randn((num_heads, seq_len, head_dim), generator=g, device=device)
    q = torch.randn((num_heads, head_dim), generator=g, device=device)
    return q.to(dtype), keys.to(dtype), values.to(dtype)
