"""Paged-KV fused decode attention (block-table gather).

Drop-in for ``orthocache_gpu.triton_kernels.paged_eviction``
(j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/paged_eviction.py).
Pages are moved whole: every 64-token tile is assembled in shared memory by
one bulk copy per page run (a 16-token page of 128 fp16 columns is one 4 KB
copy) after one block-table lookup per page, instead of 64 per-row lookups.

Cache layout (num_blocks, num_kv_heads, block_size, head_dim); block_tables
(num_seqs, max_blocks) int32.  With the defaults this is the reference's
MHA, ζ-gated, fixed-length path.  Additive keyword-only extensions:

* ``seq_lens`` (num_seqs,) int32 multiples of 64: ragged sequences;
* GQA: num_query_heads may be a multiple of num_kv_heads (query heads
  [h*G, (h+1)*G) share kv head h);
* ``tau``: use the V3 Cauchy-Schwarz gate with this threshold instead of ζ;
* ``return_mask``, ``stats`` as in V2.

float8 key caches are read natively (one byte a key element) and each
element is de-quantised in registers exactly as the reference's host-side
``k_cache.to(q.dtype) * k_scale`` would round it (paged_eviction.py:355-357),
so the gate and the logits see the same keys; the reference materialises a
de-quantised copy of the whole cache instead.
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib
from .fused_eviction import _auto_num_splits, _finish_meta
from .fwht_fused_prototype import TILE_SIZE, _check_tile_size


def fused_orthocache_attention_paged(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    zeta_max: Optional[float],
    num_splits: Optional[int] = None,
    tile_size: int = TILE_SIZE,
    k_scale: float = 1.0,
    *,
    seq_lens: Optional[torch.Tensor] = None,
    tau: Optional[float] = None,
    return_mask: bool = False,
    stats: bool = True,
) -> Tuple[torch.Tensor, Dict[str, Any]]:
    """Paged split-K decode (reference paged_eviction.py:323-445).

    q (num_seqs, num_query_heads, head_dim).  Returns (out like q in q's
    dtype, metadata).
    """
    num_seqs, num_heads, head_dim = q.shape
    num_physical_blocks = k_cache.shape[0]
    num_kv_heads = k_cache.shape[1]
    block_size = k_cache.shape[2]
    max_blocks_per_seq = block_tables.shape[1]
    num_tiles = (max_blocks_per_seq * block_size) // tile_size
    seq_len = num_tiles * tile_size
    assert (head_dim & (head_dim - 1)) == 0 and head_dim > 0, f"head_dim ({head_dim}) must be a power of 2"
    assert (tile_size & (tile_size - 1)) == 0 and tile_size > 0, f"tile_size ({tile_size}) must be a power of 2"
    assert (block_size & (block_size - 1)) == 0 and block_size > 0, f"block_size ({block_size}) must be a power of 2"
    assert (seq_len % tile_size) == 0, f"seq_len {seq_len} not divisible by tile_size {tile_size}"
    if num_splits is not None:
        assert num_splits > 0, f"num_splits ({num_splits}) must be positive"
    assert num_heads % num_kv_heads == 0, (
        f"num_query_heads ({num_heads}) must be a multiple of num_kv_heads ({num_kv_heads})")
    if tau is None and zeta_max is None:
        raise ValueError("give zeta_max (ζ gate) or tau (Cauchy-Schwarz gate)")
    _check_tile_size(tile_size)
    group = num_heads // num_kv_heads

    input_dtype = q.dtype
    fp8_keys = k_cache.dtype == torch.float8_e4m3fn
    # float8 keys are de-quantised into q's dtype inside the kernel
    # (round(k * k_scale) per element, paged_eviction.py:355-357); other
    # dtypes fold k_scale into q like the reference
    deq_scale = float(k_scale) if fp8_keys else 1.0
    if k_scale != 1.0 and not fp8_keys:
        q = q * k_scale
    dev = _lib.require_cuda(q, k_cache, v_cache, block_tables)
    if num_splits is None:
        num_splits = _auto_num_splits(num_tiles, dev)
    num_splits = max(1, min(num_splits, max(num_tiles, 1)))

    q = q if q.stride(-1) == 1 else q.contiguous()
    k_cache, v_cache = _lib.harmonize_kv(k_cache, v_cache)
    k_cache = _lib.prepare_kv(k_cache)
    v_cache = _lib.prepare_kv(v_cache)
    bt = block_tables.to(torch.int32)
    bt = bt if bt.stride(-1) == 1 else bt.contiguous()
    sl = None
    if seq_lens is not None:
        sl = seq_lens.to(device=dev, dtype=torch.int32).contiguous()
        assert sl.numel() == num_seqs, "seq_lens must have one entry per sequence"
    out = torch.empty((num_seqs, num_heads, head_dim), dtype=input_dtype, device=dev)
    # tiles beyond a sequence's length are never gated: they read False (evicted)
    mask = torch.zeros((num_seqs, num_kv_heads, num_tiles), dtype=torch.bool, device=dev) if return_mask else None

    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    wptr, wbytes = ws.get(_lib.workspace_bytes(num_seqs * num_kv_heads, group, num_tiles, head_dim))
    gate = _lib.OC_GATE_ZETA if tau is None else _lib.OC_GATE_CAUCHY_SCHWARZ
    thr = float(zeta_max) if tau is None else float(tau)
    _lib.check(_lib.load().oc_fused_attention_paged(
        q.data_ptr(), _lib.dtype_code(q), q.stride(0), q.stride(1),
        k_cache.data_ptr(), _lib.dtype_code(k_cache), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.data_ptr(), _lib.dtype_code(v_cache), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        num_physical_blocks, block_size, bt.data_ptr(), bt.stride(0), max_blocks_per_seq, _lib.ptr(sl),
        num_seqs, num_kv_heads, group, head_dim, gate, thr, deq_scale, num_splits, _lib.num_sms(dev),
        out.data_ptr(), _lib.dtype_code(out), out.stride(0), out.stride(1),
        _lib.ptr(mask), ws.retained_ptr if stats else 0, ws.status_ptr,
        wptr, wbytes, stream), "fused_orthocache_attention_paged")

    meta: Dict[str, Any] = {
        "num_splits": num_splits,
        "num_tiles": num_tiles,
        "num_heads": num_heads,
        "num_seqs": num_seqs,
        "layout": "paged",
        "tile_assignment": "contiguous",
        "gate_type": "zeta" if tau is None else "cauchy_schwarz",
    }
    if return_mask:
        meta["eviction_mask"] = mask
    if stats:
        total = num_tiles * num_kv_heads * num_seqs
        if sl is not None:
            total = int((sl // tile_size).clamp(max=num_tiles).sum().item()) * num_kv_heads
        _finish_meta(meta, ws, total, True)
    else:
        meta["status"] = ws.status
    return out, meta
