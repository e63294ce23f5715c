"""O(1) decode gate from cached key norms, and decode attention that skips evicted tiles entirely.

Drop-in for ``orthocache_gpu.triton_kernels.decode_gate``
(j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/decode_gate.py).
During decoding the key cache is static, so the gate reads one cached
|K_high|_F per tile (``SpectralNormCache``) instead of the tile:

    evict[h, t] = s_h * |K_high|_F[h, t] <= tau * (64 * head_dim)

with s_h the max over the kv head's query heads of |q_high|_2 (``tight``,
the exact block-sum projection of ``compute_q_high_norm_exact``) or of |q|_2.
True = EVICT in this module (decode_gate.py:199), the opposite polarity of
the ζ / Cauchy-Schwarz masks.  The reference's GPU (Triton) kernel uses the
loose |q|_2 (decode_gate.py:148-164) while its PyTorch path defaults to the
tight norm (:251-300); ``tight`` selects either, default tight.

``fused_orthocache_attention_cached`` gates and then decodes over the
retained tiles only, so an evicted tile costs neither its K nor its V read.
The reference applies the same gate inside its model hook by masking the
logits of a dense product (eval/perplexity_eval.py:554-674; its median
statistic is ``q_stat='median'``).
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib
from .fused_eviction import _finish_meta
from .fwht_fused_prototype import TILE_SIZE

_Q_STAT = {"max": 0, "median": 1}


def compute_q_high_norm_exact(q: torch.Tensor, low_band: int = 8) -> torch.Tensor:
    """|q_high|_2 = sqrt(max(0, |q|^2 - sum_i S_i^2 / bs)) over the last dim (decode_gate.py:54-106).

    S_i are the sums of ``low_band`` contiguous blocks of bs = head_dim /
    low_band dims.  A few element-wise tensor ops on q's device (the gate
    kernel evaluates the same formula in registers).
    """
    head_dim = q.shape[-1]
    block_size = head_dim // low_band
    assert head_dim % low_band == 0, f"head_dim ({head_dim}) must be divisible by low_band ({low_band})"
    qf = q.float()
    q_norm_sq = (qf * qf).sum(dim=-1)
    bsum = qf.reshape(*qf.shape[:-1], low_band, block_size).sum(dim=-1)
    q_low_sq = (bsum * bsum).sum(dim=-1) / block_size
    return torch.sqrt(torch.clamp(q_norm_sq - q_low_sq, min=0.0))


def _norm_tensor(norm_cache):
    return norm_cache.cache if hasattr(norm_cache, "cache") else norm_cache


def decode_gate(q: torch.Tensor, norm_cache, tau: float, num_tiles: int, G: int, tile_size: int = TILE_SIZE,
                *, tight: bool = True, q_stat: str = "max", low_band: int = 8) -> Tuple[torch.Tensor, torch.Tensor]:
    """Eviction mask from cached norms (decode_gate.py:188-300).

    q (num_q_heads, head_dim); norm_cache (num_kv_heads, max_tiles) float32
    (or a ``SpectralNormCache``).  Returns (evict (num_kv_heads, max_tiles)
    bool, True = evict, False beyond ``num_tiles``; q_norms (num_kv_heads,)
    float32, the statistic s_h).
    """
    nc = _norm_tensor(norm_cache)
    num_q_heads, head_dim = q.shape
    assert num_q_heads % G == 0, f"num_query_heads ({num_q_heads}) must be a multiple of G ({G})"
    num_kv_heads = num_q_heads // G
    max_tiles = nc.shape[1]
    assert nc.shape[0] >= num_kv_heads and 0 <= num_tiles <= max_tiles
    if tile_size != TILE_SIZE:
        raise NotImplementedError(f"tile_size={tile_size}: the gate implements 64-token tiles")
    dev = _lib.require_cuda(q, nc)
    nc = nc if (nc.dtype == torch.float32 and nc.stride(-1) == 1) else nc.float().contiguous()
    q = q if q.stride(-1) == 1 else q.contiguous()
    mask = torch.empty((num_kv_heads, max_tiles), dtype=torch.bool, device=dev)
    q_norms = torch.empty(num_kv_heads, dtype=torch.float32, device=dev)
    _lib.check(_lib.load().oc_decode_gate(
        q.data_ptr(), _lib.dtype_code(q), q.stride(0), num_kv_heads, G, head_dim, nc.data_ptr(), nc.stride(0),
        num_tiles, max_tiles, float(tau), int(tight), low_band, _Q_STAT[q_stat], mask.data_ptr(),
        q_norms.data_ptr(), _lib.stream_ptr(dev)), "decode_gate")
    return mask, q_norms


def apply_decode_mask_vectorized(logits: torch.Tensor, mask: torch.Tensor, G: int, tile_size: int = TILE_SIZE,
                                 num_tiles: Optional[int] = None) -> torch.Tensor:
    """Set the logits (num_q_heads, 1, seq_len) of evicted tiles to -inf (decode_gate.py:345-383)."""
    num_kv_heads = mask.shape[0]
    seq_len_kv = logits.shape[2]
    if num_tiles is None:
        num_tiles = seq_len_kv // tile_size
    tok = mask[:, :num_tiles, None].expand(num_kv_heads, num_tiles, tile_size).reshape(num_kv_heads, -1)
    if tok.shape[1] < seq_len_kv:
        tok = torch.cat([tok, tok.new_zeros(num_kv_heads, seq_len_kv - tok.shape[1])], 1)
    tok = tok[:, :seq_len_kv].repeat_interleave(G, dim=0)
    logits[:, 0, :][tok] = float("-inf")
    return logits


apply_decode_mask = apply_decode_mask_vectorized  # same result as the reference's looped form (:309-342)


def _cached_call(q, keys, values, norm_cache, tau, G, tight, q_stat, return_mask, stats, states):
    batched = keys.ndim == 4
    num_kv_heads, seq_len, head_dim = keys.shape[-3:]
    num_tiles = seq_len // TILE_SIZE
    assert seq_len == num_tiles * TILE_SIZE, f"seq_len {seq_len} not divisible by tile_size {TILE_SIZE}"
    assert q.shape[-2] == num_kv_heads * G, (
        f"num_query_heads ({q.shape[-2]}) != num_kv_heads ({num_kv_heads}) × G ({G})")
    nc = _norm_tensor(norm_cache)
    if not batched:
        q, keys, values, nc = q.unsqueeze(0), keys.unsqueeze(0), values.unsqueeze(0), nc.unsqueeze(0)
    num_seqs = keys.shape[0]
    assert nc.shape[-2] >= num_kv_heads and nc.shape[-1] >= num_tiles and nc.shape[0] == num_seqs
    input_dtype = q.dtype
    dev = _lib.require_cuda(q, keys, values, nc)
    nc = nc if (nc.dtype == torch.float32 and nc.stride(-1) == 1) else nc.float().contiguous()
    q = q if q.stride(-1) == 1 else q.contiguous()
    keys, values = _lib.harmonize_kv(keys, values)
    keys, values = _lib.prepare_kv(keys), _lib.prepare_kv(values)
    hq = num_kv_heads * G
    if states:
        m = torch.empty((num_seqs, hq), dtype=torch.float32, device=dev)
        l = torch.empty_like(m)
        acc = torch.empty((num_seqs, hq, head_dim), dtype=torch.float32, device=dev)
        out, optr, st = None, 0, (m.data_ptr(), l.data_ptr(), acc.data_ptr())
    else:
        out = torch.empty((num_seqs, hq, head_dim), dtype=input_dtype, device=dev)
        optr, st = out.data_ptr(), (0, 0, 0)
    mask = torch.empty((num_seqs, num_kv_heads, num_tiles), dtype=torch.bool, device=dev) if return_mask else None
    q_norms = torch.empty((num_seqs, num_kv_heads), dtype=torch.float32, device=dev) if return_mask else None
    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    wptr, wbytes = ws.get(_lib.load().oc_cached_workspace_bytes(num_seqs * num_kv_heads, G, num_tiles, head_dim))
    _lib.check(_lib.load().oc_fused_attention_cached(
        q.data_ptr(), _lib.dtype_code(q), q.stride(0), q.stride(1),
        keys.data_ptr(), _lib.dtype_code(keys), keys.stride(0), keys.stride(1), keys.stride(2),
        values.data_ptr(), _lib.dtype_code(values), values.stride(0), values.stride(1), values.stride(2),
        num_seqs, num_kv_heads, G, seq_len, head_dim, nc.data_ptr(), nc.stride(0), nc.stride(1),
        float(tau), int(tight), _Q_STAT[q_stat], _lib.num_sms(dev),
        optr, _lib.dtype_code(q), hq * head_dim, head_dim, *st,
        _lib.ptr(mask), _lib.ptr(q_norms), ws.retained_ptr if stats else 0, ws.status_ptr,
        wptr, wbytes, stream), "fused_orthocache_attention_cached")
    res = (m, l, acc) if states else (out,)
    if not batched:
        res = tuple(t[0] for t in res)
        if mask is not None:
            mask, q_norms = mask[0], q_norms[0]
    meta: Dict[str, Any] = {"num_tiles": num_tiles, "num_kv_heads": num_kv_heads, "num_query_groups": G,
                            "gate_type": "cached_norm", "tight": tight, "q_stat": q_stat}
    if batched:
        meta["num_seqs"] = num_seqs
    if return_mask:
        meta["evict_mask"] = mask
        meta["q_norms"] = q_norms
    return res, _finish_meta(meta, ws, num_tiles * num_kv_heads * num_seqs, stats)


def fused_orthocache_attention_cached(
    q: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    norm_cache,
    tau: float,
    num_query_groups: int,
    *,
    tight: bool = True,
    q_stat: str = "max",
    return_mask: bool = False,
    stats: bool = True,
) -> Tuple[torch.Tensor, Dict[str, Any]]:
    """Decode attention over the tiles the cached-norm gate retains.

    q (Hq, hd); keys / values (KVH, S, hd), or with a leading batch on all
    three; norm_cache (KVH, >= S/64) float32, (B, KVH, >= S/64) when
    batched, or a ``SpectralNormCache`` whose first S/64 tiles are valid.
    Returns (out like q in q's dtype, metadata); ``meta['evict_mask']``
    (with ``return_mask``) is the gate's mask, True = evicted.
    """
    (out,), meta = _cached_call(q, keys, values, norm_cache, tau, num_query_groups, tight, q_stat, return_mask,
                                stats, False)
    return out, meta


def cached_partials(q, keys, values, norm_cache, tau: float, num_query_groups: int, *, tight: bool = True,
                    q_stat: str = "max", stats: bool = False):
    """Like ``fused_orthocache_attention_cached`` but returns each query head's merged softmax state.

    Returns ((m, l, acc), meta): float32 m, l (..., Hq) with m in log2 units
    and acc (..., Hq, hd) unnormalised, for a log-sum-exp merge with other
    partial states (a ragged tail of tokens, other sequence shards).
    """
    return _cached_call(q, keys, values, norm_cache, tau, num_query_groups, tight, q_stat, False, stats, True)
