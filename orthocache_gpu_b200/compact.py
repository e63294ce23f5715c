"""512-token block compaction mode of ``orthocache_forward`` (``mode='compact'``).

Host code around one kernel launch, after the reference pipeline
(j-arndt/orthocache-gpu, src/orthocache_gpu/pipeline.py:459-555):

1. spectral analysis of every 512-token block of every head with a 512-point
   natural-order Walsh-Hadamard transform along the tokens (1/sqrt(512)
   normalised; spectral_energy.py:20-238, fwht.py:5-66): band energies, the
   spectral decay ratio ζ = E_high / (E_low + 1e-6) with bands [1, 64) and
   [256, 512), and the query-aware logit bound DC alignment + |q| sqrt(E_AC)
   / sqrt(hd);
2. the two-gate mask (bound >= tau for some query AND ζ <= zeta_max), tau
   defaulting to mean - std of the per-block bounds, unified over heads;
3. the perfect-eviction classification of evicted blocks
   (perfect_eviction.py:75-187) for the metadata;
4. attention of every query position over the retained blocks only -- the
   library's kernel over the retained blocks' 64-token tiles (a tile list
   shared by all heads), so evicted blocks are never read.  Like the
   reference (adaptive_attention.py:159-205) the attention is not causal and
   the output is bfloat16.

Steps 1-3 are PyTorch tensor code on the inputs' device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from .fused_eviction import _finish_meta

BAND_DC = 0
BAND_LOW = (1, 64)
BAND_MID = (64, 256)
BAND_HIGH = (256, 512)
FLOAT32_UNDERFLOW_THRESHOLD = 88.72
BFLOAT16_UNDERFLOW_THRESHOLD = 87.34


def fwht_512(x: torch.Tensor) -> torch.Tensor:
    """512-point natural-order Walsh-Hadamard transform along dim 0, / sqrt(512) (fwht.py:5-66)."""
    n = 512
    one_d = x.ndim == 1
    y = x[:, None] if one_d else x
    d = y.shape[1]
    h = 1
    while h < n:
        y = y.reshape(n // (2 * h), 2, h, d)
        y = torch.stack((y[:, 0] + y[:, 1], y[:, 0] - y[:, 1]), dim=1)
        h *= 2
    y = y.reshape(n, d) / math.sqrt(n)
    return y[:, 0] if one_d else y


def _spectral_blocks(keys: torch.Tensor, block_size: int) -> torch.Tensor:
    """(num_blocks, block_size, heads, hd) Walsh coefficients of each block along its tokens."""
    seq, heads, hd = keys.shape
    nb = seq // block_size
    assert block_size == 512, "the block transform is 512-point"
    t = keys[: nb * block_size].reshape(nb, block_size, heads, hd).permute(1, 0, 2, 3).reshape(block_size, -1)
    return fwht_512(t).reshape(block_size, nb, heads, hd).permute(1, 0, 2, 3)


def compute_block_energy(keys: torch.Tensor, block_size: int = 512) -> torch.Tensor:
    """Sum of squared keys per (block, head) (spectral_energy.py:20-34)."""
    seq, heads, hd = keys.shape
    nb = seq // block_size
    return torch.sum(keys[: nb * block_size].reshape(nb, block_size, heads, hd) ** 2, dim=(1, 3))


def compute_spectral_bands(keys, block_size: int = 512, band_low=BAND_LOW, band_mid=BAND_MID, band_high=BAND_HIGH):
    """(dc, low, mid, high) energies per (block, head) (spectral_energy.py:68-105)."""
    s = _spectral_blocks(keys, block_size)
    e = lambda b: torch.sum(s[:, b[0]:b[1]] ** 2, dim=(1, 3))  # noqa: E731
    return s[:, BAND_DC], e(band_low), e(band_mid), e(band_high)


def compute_spectral_decay_ratio(keys, block_size: int = 512, band_low=BAND_LOW, band_high=BAND_HIGH):
    """ζ = E_high / (E_low + 1e-6) per (block, head) (spectral_energy.py:108-137)."""
    _, low, _, high = compute_spectral_bands(keys, block_size, band_low, (band_low[1], band_high[0]), band_high)
    return high / (low + 1e-6)


def compute_query_aware_bounds(q, keys, block_size: int = 512):
    """Logit upper bound per (query, block, head) (spectral_energy.py:140-176)."""
    hd = keys.shape[2]
    s = _spectral_blocks(keys, block_size)
    ac = torch.sum(s[:, 1:] ** 2, dim=(1, 3))
    mean = s[:, 0] / torch.sqrt(torch.tensor(float(block_size)))
    sq = torch.sqrt(torch.tensor(float(hd)))
    align = torch.einsum("qhd,bhd->qbh", q, mean) / sq
    resid = torch.linalg.norm(q, dim=-1)[:, None, :] * torch.sqrt(ac)[None] / sq
    return align + resid


def compute_query_aware_mask(q, keys, tau: float, block_size: int = 512):
    return torch.max(compute_query_aware_bounds(q, keys, block_size), dim=0).values >= tau


def compute_multiband_mask(q, keys, tau: float, zeta_max: float, block_size: int = 512):
    """Retain a (block, head) iff its bound >= tau AND ζ <= zeta_max (spectral_energy.py:198-233)."""
    return compute_query_aware_mask(q, keys, tau, block_size) & (compute_spectral_decay_ratio(keys, block_size)
                                                                   <= zeta_max)


def auto_tau(q, keys, block_size: int = 512) -> float:
    """mean - std of the per-block maximum bounds (pipeline.py:571-583)."""
    b = torch.max(compute_query_aware_bounds(q, keys, block_size), dim=0).values
    return float(torch.mean(b) - torch.std(b))


@dataclass
class EvictionMetadata:
    """Per-block eviction classification (perfect_eviction.py:64-73)."""
    regime: torch.Tensor
    beta: torch.Tensor
    logit_gap: torch.Tensor
    num_perfect: int
    num_statistical: int
    num_retained: int
    underflow_threshold: float


def compute_block_beta(q, block_energies, head_dim: int):
    """β = max_pos |q| sqrt(E) / sqrt(hd) per (block, head) (perfect_eviction.py:75-104)."""
    qn = torch.max(torch.linalg.norm(q.float(), dim=-1), dim=0).values
    return qn[None, :] * torch.sqrt(block_energies.float().clamp(min=0)) / math.sqrt(head_dim)


def classify_eviction(q, block_energies, z_max, block_mask, head_dim: int, accumulator_dtype: str = "float32"):
    """Perfect (gap >= underflow threshold) or statistical eviction per evicted block (perfect_eviction.py:107-186)."""
    thr = BFLOAT16_UNDERFLOW_THRESHOLD if accumulator_dtype == "bfloat16" else FLOAT32_UNDERFLOW_THRESHOLD
    beta = torch.max(compute_block_beta(q, block_energies, head_dim), dim=-1).values
    zm = torch.max(z_max).item() if isinstance(z_max, torch.Tensor) and z_max.ndim > 0 else float(z_max)
    gap = zm - beta
    keep = torch.any(block_mask, dim=-1) if block_mask.ndim > 1 else block_mask
    regime = torch.zeros(keep.shape[0], dtype=torch.int32, device=q.device)
    perfect = ~keep & (gap >= thr)
    stat = ~keep & (gap < thr)
    regime[perfect] = 1
    regime[stat] = 2
    return EvictionMetadata(regime, beta, gap, int(perfect.sum()), int(stat.sum()), int(keep.sum()), thr)


def stream_compact(block_mask: torch.Tensor):
    """(indices with the retained blocks first, in order; number retained) (adaptive_attention.py:29-42)."""
    nb = block_mask.shape[0]
    iota = torch.arange(nb, dtype=torch.int32, device=block_mask.device)
    order = torch.argsort(torch.where(block_mask, iota, nb + iota), stable=True)
    return order, int(block_mask.sum().item())


def block_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, block_mask: torch.Tensor,
                    block_size: int = 512):
    """Attention of every query over the retained blocks (adaptive_attention.py:159-205).

    q (seq_q, heads, hd); keys / values (seq_k, heads, hd); block_mask
    (num_blocks,) bool, True = keep.  One launch of the library's kernel over
    the tiles of the retained blocks (the query positions of a head form its
    query group).  Returns (output (seq_q, heads, hd) bfloat16, stats).
    """
    seq_q, heads, hd = q.shape
    seq_k = keys.shape[0]
    nb = seq_k // block_size
    order, n_act = stream_compact(block_mask)
    if n_act == 0:
        return torch.zeros_like(q), {"num_active": 0, "eviction_rate": 1.0, "path": "zero"}
    dev = _lib.require_cuda(q, keys, values)
    tpb = block_size // 64
    tiles = (order[:n_act, None].to(torch.int32) * tpb + torch.arange(tpb, device=dev, dtype=torch.int32)).reshape(-1)
    counts = torch.full((heads,), tiles.numel(), dtype=torch.int32, device=dev)
    qh = q.permute(1, 0, 2).contiguous()                           # (heads, seq_q, hd): kv head h, group seq_q
    kv_len = nb * block_size
    k, v = _lib.harmonize_kv(keys[:kv_len], values[:kv_len])
    k, v = _lib.prepare_kv(k), _lib.prepare_kv(v)
    out = torch.empty((heads, seq_q, hd), dtype=torch.bfloat16, device=dev)
    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    lib = _lib.load()
    # at most 2048 (head, chunk of 8 query positions) units per launch
    qmax = max(8, (2048 // heads) * 8)
    for s0 in range(0, seq_q, qmax):
        g = min(qmax, seq_q - s0)
        whole = g == seq_q
        qc = qh if whole else qh[:, s0:s0 + g].contiguous()
        oc_ = out if whole else torch.empty((heads, g, hd), dtype=torch.bfloat16, device=dev)
        wptr, wbytes = ws.get(_lib.workspace_bytes(heads, g, nb * tpb, hd))
        _lib.check(lib.oc_fused_attention_tiles(
            qc.data_ptr(), _lib.dtype_code(qc), 0, hd,
            k.data_ptr(), _lib.dtype_code(k), 0, k.stride(1), k.stride(0),
            v.data_ptr(), _lib.dtype_code(v), 0, v.stride(1), v.stride(0),
            1, heads, g, kv_len, hd, tiles.data_ptr(), 0, counts.data_ptr(), _lib.num_sms(dev),
            oc_.data_ptr(), _lib.OC_BF16, 0, hd, 0, 0, 0, 0, ws.status_ptr, wptr, wbytes, stream), "block_attention")
        if not whole:
            out[:, s0:s0 + g] = oc_
    return out.permute(1, 0, 2), {"num_active": n_act, "num_blocks": nb, "eviction_rate": 1.0 - n_act / nb,
                                  "path": "fused_tiles"}


def compact_forward(q, keys, values, block_size, zeta_max, tau, metadata):
    """The compact branch of orthocache_forward (pipeline.py:459-555); fills ``metadata``."""
    import time
    head_dim = keys.shape[2]
    num_blocks = keys.shape[0] // block_size
    t0 = time.perf_counter()
    zeta = compute_spectral_decay_ratio(keys, block_size)
    if tau is None:
        tau = auto_tau(q, keys, block_size)
        metadata["tau_auto"] = True
    else:
        metadata["tau_auto"] = False
    metadata["tau"] = tau
    block_mask = compute_multiband_mask(q, keys, tau, zeta_max, block_size)
    t1 = time.perf_counter()
    metadata["spectral_ms"] = (t1 - t0) * 1000
    za = torch.mean(zeta, dim=-1)
    metadata["zeta_mean"] = float(torch.mean(za))
    metadata["zeta_std"] = float(torch.std(za))
    metadata["zeta_min"] = float(torch.min(za))
    metadata["zeta_max_observed"] = float(torch.max(za))
    unified = torch.any(block_mask, dim=-1)
    kept = int(unified.sum())
    metadata["blocks_retained"] = kept
    metadata["blocks_evicted"] = num_blocks - kept
    metadata["eviction_rate"] = float(1.0 - kept / num_blocks)
    energies = compute_block_energy(keys, block_size)
    with torch.no_grad():
        if unified.any():
            mb = torch.max(compute_query_aware_bounds(q, keys, block_size), dim=0).values
            z_max = torch.max(mb[unified])
        else:
            z_max = torch.tensor(0.0, device=q.device)
    em = classify_eviction(q, energies, z_max, block_mask, head_dim)
    metadata["perfect_eviction_blocks"] = em.num_perfect
    metadata["statistical_eviction_blocks"] = em.num_statistical
    metadata["perfect_eviction_rate"] = (em.num_perfect / max(1, num_blocks - kept)) if num_blocks > kept else 0.0
    t2 = time.perf_counter()
    out, _ = block_attention(q, keys, values, unified, block_size)
    metadata["compact_num_active"] = kept
    t3 = time.perf_counter()
    metadata["attention_ms"] = (t3 - t2) * 1000
    metadata["total_ms"] = (t3 - t0) * 1000
    return out, metadata
