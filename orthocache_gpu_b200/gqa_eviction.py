"""V3: GQA decode attention with the Cauchy-Schwarz spectral gate.

Drop-in for ``orthocache_gpu.triton_kernels.gqa_eviction``
(j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/gqa_eviction.py).
One CTA per (kv head, split) scores each tile once for the whole query
group: a tile is evicted iff max_g(|q_g|_2 * |K_high|_F) <= tau, where
|K_high|_F^2 is the energy of natural-order Walsh rows [32, 64) of the tile
(gqa_eviction.py:216-239, norms below 1e-38 read as 0).  The G query heads'
online-softmax states live in registers, not in HBM.

Additive extensions: an optional leading batch dimension (q (B, Hq, hd),
keys / values (B, KVH, S, hd)), keyword-only ``return_mask`` and ``stats``.
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib
from .fused_eviction import _auto_num_splits, _finish_meta
from .fwht_fused_prototype import TILE_SIZE, _check_tile_size


def _auto_num_splits_gqa(num_tiles: int, device: torch.device) -> int:
    """Same heuristic as V2 (gqa_eviction.py:502-508)."""
    return _auto_num_splits(num_tiles, device)


def fused_orthocache_attention_v3_gqa(
    q: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    tau: float,
    num_query_groups: int,
    num_splits: Optional[int] = None,
    tile_size: int = TILE_SIZE,
    k_scale: float = 1.0,
    *,
    return_mask: bool = False,
    stats: bool = True,
) -> Tuple[torch.Tensor, Dict[str, Any]]:
    """GQA Cauchy-Schwarz split-K decode (reference gqa_eviction.py:511-639).

    q (num_query_heads, head_dim), query heads [g*G, (g+1)*G) sharing kv
    head g; keys / values (num_kv_heads, seq_len, head_dim).  With a leading
    batch dimension on all three, every batch element is an independent
    sequence.  Returns (out like q in q's dtype, metadata).
    """
    batched = keys.ndim == 4
    num_kv_heads, seq_len, head_dim = keys.shape[-3:]
    num_query_heads = q.shape[-2]
    G = num_query_groups
    num_tiles = seq_len // tile_size
    assert (head_dim & (head_dim - 1)) == 0 and head_dim > 0, f"head_dim ({head_dim}) must be a power of 2"
    assert (tile_size & (tile_size - 1)) == 0 and tile_size > 0, f"tile_size ({tile_size}) must be a power of 2"
    assert num_query_heads == num_kv_heads * G, (
        f"num_query_heads ({num_query_heads}) != num_kv_heads ({num_kv_heads}) × G ({G})")
    assert seq_len == num_tiles * tile_size, f"seq_len {seq_len} not divisible by tile_size {tile_size}"
    if num_splits is not None:
        assert num_splits > 0, f"num_splits ({num_splits}) must be greater than 0"
    _check_tile_size(tile_size)

    input_dtype = q.dtype
    if k_scale != 1.0:
        q = q * k_scale
    dev = _lib.require_cuda(q, keys, values)
    if num_splits is None:
        num_splits = _auto_num_splits_gqa(num_tiles, dev)
    num_splits = max(1, min(num_splits, max(num_tiles, 1)))

    if not batched:
        q, keys, values = q.unsqueeze(0), keys.unsqueeze(0), values.unsqueeze(0)
    num_seqs = keys.shape[0]
    assert q.shape[0] == num_seqs and values.shape[:3] == keys.shape[:3], "batch / head shapes of q, keys, values differ"
    q = q if q.stride(-1) == 1 else q.contiguous()
    keys, values = _lib.harmonize_kv(keys, values)
    keys = _lib.prepare_kv(keys)
    values = _lib.prepare_kv(values)
    mask = torch.empty((num_seqs, num_kv_heads, num_tiles), dtype=torch.bool, device=dev) if return_mask else None

    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    wptr, wbytes = ws.get(_lib.workspace_bytes(num_seqs * num_kv_heads, G, num_tiles, head_dim))
    fast = _lib.binding()
    if fast is not None:
        out = fast.v3(q, keys, values, float(tau), G, num_splits, _lib.num_sms(dev), input_dtype, mask,
                      ws.retained_ptr if stats else 0, ws.status_ptr, wptr, wbytes, stream)
    else:
        out = torch.empty((num_seqs, num_query_heads, head_dim), dtype=input_dtype, device=dev)
        _lib.check(_lib.load().oc_fused_attention_v3_gqa(
            q.data_ptr(), _lib.dtype_code(q), q.stride(0), q.stride(1),
            keys.data_ptr(), _lib.dtype_code(keys), keys.stride(0), keys.stride(1), keys.stride(2),
            values.data_ptr(), _lib.dtype_code(values), values.stride(0), values.stride(1), values.stride(2),
            num_seqs, num_kv_heads, G, seq_len, head_dim, float(tau), num_splits, _lib.num_sms(dev),
            out.data_ptr(), _lib.dtype_code(out), out.stride(0), out.stride(1),
            _lib.ptr(mask), ws.retained_ptr if stats else 0, ws.status_ptr,
            wptr, wbytes, stream), "fused_orthocache_attention_v3_gqa")

    if not batched:
        out = out[0]
        if mask is not None:
            mask = mask[0]
    meta: Dict[str, Any] = {
        "num_splits": num_splits,
        "num_tiles": num_tiles,
        "num_kv_heads": num_kv_heads,
        "num_query_heads": num_query_heads,
        "num_query_groups": G,
        "tile_assignment": "interleaved",
        "gate_type": "cauchy_schwarz",
    }
    if batched:
        meta["num_seqs"] = num_seqs
    if return_mask:
        meta["eviction_mask"] = mask
    return out, _finish_meta(meta, ws, num_tiles * num_kv_heads * num_seqs, stats)
