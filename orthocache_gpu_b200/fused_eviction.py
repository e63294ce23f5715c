"""ζ-gated fused decode attention: V1 (single head) and V2 (split-K multi-head).

Drop-in for ``orthocache_gpu.triton_kernels.fused_eviction``
(j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/fused_eviction.py):
same signatures, argument meaning, assertion messages and output dtype.  One
launch of the library's sm_100a kernel scores every 64-token K tile,
streams V only for retained tiles, and merges the split-K partials in the
same launch.

Differences from the reference, all additive:

* keyword-only ``return_mask`` on V2 (V1 already has it);
* keyword-only ``stats`` (default True): the metadata carries
  ``tiles_retained`` / ``tiles_evicted`` / ``eviction_rate`` (the reference's
  CPU-path keys) next to the GPU-path keys, read back with one synchronising
  copy that also raises if the kernel reported an error.  ``stats=False``
  skips that read (no host synchronisation at all, e.g. for CUDA-graph
  capture) and puts the device status word in ``meta['status']`` instead;
  ``check_status()`` raises on it later;
* strided keys / values are streamed in place instead of being copied by
  ``.contiguous()`` when their rows are 16-byte aligned.
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib
from .fwht_fused_prototype import TILE_SIZE, _check_tile_size


def _auto_num_splits(num_tiles: int, device: torch.device) -> int:
    """The reference's split heuristic (fused_eviction.py:556-570)."""
    if device.type != "cuda":
        return 1
    return _lib.auto_num_splits(num_tiles, device)


def _finish_meta(meta: Dict[str, Any], ws, num_tiles_total: int, stats: bool) -> Dict[str, Any]:
    """Add the counts (one synchronising read) or, with ``stats=False``, the device status word.

    Without stats nothing is read back: ``meta['status']`` is the stream's
    sticky status word on the device (0 = every launch so far was valid);
    ``orthocache_gpu_b200.check_status()`` reads it and raises.
    """
    if stats:
        kept = _lib.read_stats(ws)
        meta["tiles_retained"] = kept
        meta["tiles_evicted"] = num_tiles_total - kept
        meta["eviction_rate"] = (num_tiles_total - kept) / max(1, num_tiles_total)
    else:
        meta["status"] = ws.status
    return meta


def fused_orthocache_attention_v2(
    q: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    zeta_max: float,
    num_splits: Optional[int] = None,
    tile_size: int = TILE_SIZE,
    k_scale: float = 1.0,
    *,
    return_mask: bool = False,
    stats: bool = True,
) -> Tuple[torch.Tensor, Dict[str, Any]]:
    """Multi-head ζ-gated split-K decode attention (reference fused_eviction.py:573-691).

    q (num_heads, head_dim); keys / values (num_heads, seq_len, head_dim).
    A 64-token tile is evicted iff ζ > zeta_max; evicted tiles contribute
    nothing and their V is never read.  Returns (out (num_heads, head_dim)
    in q's dtype, metadata).
    """
    num_heads = q.shape[0]
    head_dim = q.shape[-1]
    seq_len = keys.shape[1]
    num_tiles = seq_len // tile_size
    assert (head_dim & (head_dim - 1)) == 0 and head_dim > 0, f"head_dim ({head_dim}) must be a power of 2"
    assert (tile_size & (tile_size - 1)) == 0 and tile_size > 0, f"tile_size ({tile_size}) must be a power of 2"
    assert seq_len == num_tiles * tile_size, f"seq_len {seq_len} not divisible by tile_size {tile_size}"
    if num_splits is not None:
        assert num_splits > 0, f"num_splits ({num_splits}) must be greater than 0"
    _check_tile_size(tile_size)

    input_dtype = q.dtype
    if k_scale != 1.0:
        q = q * k_scale
    dev = _lib.require_cuda(q, keys, values)
    if num_splits is None:
        num_splits = _auto_num_splits(num_tiles, dev)
    num_splits = max(1, min(num_splits, max(num_tiles, 1)))

    q = q if q.stride(-1) == 1 else q.contiguous()
    keys, values = _lib.harmonize_kv(keys, values)
    keys = _lib.prepare_kv(keys)
    values = _lib.prepare_kv(values)
    mask = torch.empty((num_heads, num_tiles), dtype=torch.bool, device=dev) if return_mask else None

    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    wptr, wbytes = ws.get(_lib.workspace_bytes(num_heads, 1, num_tiles, head_dim))
    fast = _lib.binding()
    if fast is not None:
        out = fast.v2(q, keys, values, float(zeta_max), num_splits, _lib.num_sms(dev), input_dtype, mask,
                      ws.retained_ptr if stats else 0, ws.status_ptr, wptr, wbytes, stream)
    else:
        out = _v2_ctypes(q, keys, values, zeta_max, num_splits, dev, input_dtype, mask, ws, stats, wptr, wbytes,
                         stream)
    meta: Dict[str, Any] = {
        "num_splits": num_splits,
        "num_tiles": num_tiles,
        "num_heads": num_heads,
        "tile_assignment": "interleaved",
    }
    if return_mask:
        meta["eviction_mask"] = mask
    return out, _finish_meta(meta, ws, num_tiles * num_heads, stats)


def _v2_ctypes(q, keys, values, zeta_max, num_splits, dev, input_dtype, mask, ws, stats, wptr, wbytes, stream):
    """The V2 launch through ctypes (when the compiled binding is not in use)."""
    num_heads, head_dim = q.shape[0], q.shape[-1]
    seq_len = keys.shape[1]
    out = torch.empty((num_heads, head_dim), dtype=input_dtype, device=dev)
    _lib.check(_lib.load().oc_fused_attention_v2(
        q.data_ptr(), _lib.dtype_code(q), q.stride(0),
        keys.data_ptr(), _lib.dtype_code(keys), keys.stride(0), keys.stride(1),
        values.data_ptr(), _lib.dtype_code(values), values.stride(0), values.stride(1),
        num_heads, seq_len, head_dim, float(zeta_max), num_splits, _lib.num_sms(dev),
        out.data_ptr(), _lib.dtype_code(out), out.stride(0),
        _lib.ptr(mask), ws.retained_ptr if stats else 0, ws.status_ptr,
        wptr, wbytes, stream), "fused_orthocache_attention_v2")
    return out


def fused_orthocache_attention(
    q: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    zeta_max: float,
    tile_size: int = TILE_SIZE,
    return_mask: bool = False,
    k_scale: float = 1.0,
    *,
    stats: bool = True,
) -> Tuple[torch.Tensor, Dict[str, Any]]:
    """Single-query ζ-gated decode attention (reference fused_eviction.py:698-800).

    q (1, head_dim); keys / values (num_tiles*tile_size, head_dim).
    ``return_mask`` adds ``eviction_mask`` (num_tiles,) bool, True = retained.
    The reference runs this on one CTA; here it is split across the GPU.
    """
    assert q.ndim == 2 and q.shape[0] == 1, f"q must be (1, head_dim), got {q.shape}"
    head_dim = q.shape[-1]
    num_tokens = keys.shape[0]
    num_tiles = num_tokens // tile_size
    assert (head_dim & (head_dim - 1)) == 0 and head_dim > 0, f"head_dim ({head_dim}) must be a power of 2"
    assert (tile_size & (tile_size - 1)) == 0 and tile_size > 0, f"tile_size ({tile_size}) must be a power of 2"
    assert num_tokens == num_tiles * tile_size, f"seq_len {num_tokens} not divisible by tile_size {tile_size}"
    _check_tile_size(tile_size)

    input_dtype = q.dtype
    if k_scale != 1.0:
        q = q * k_scale
    dev = _lib.require_cuda(q, keys, values)
    q = q.contiguous()
    keys, values = _lib.harmonize_kv(keys, values)
    keys = _lib.prepare_kv(keys)
    values = _lib.prepare_kv(values)
    out = torch.empty((1, head_dim), dtype=input_dtype, device=dev)
    mask = torch.empty(num_tiles, dtype=torch.bool, device=dev) if return_mask else None

    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    wptr, wbytes = ws.get(_lib.workspace_bytes(1, 1, num_tiles, head_dim))
    _lib.check(_lib.load().oc_fused_attention_v1(
        q.data_ptr(), _lib.dtype_code(q),
        keys.data_ptr(), _lib.dtype_code(keys), keys.stride(0),
        values.data_ptr(), _lib.dtype_code(values), values.stride(0),
        num_tokens, head_dim, float(zeta_max), _lib.num_sms(dev),
        out.data_ptr(), _lib.dtype_code(out),
        _lib.ptr(mask), ws.retained_ptr if stats else 0, ws.status_ptr,
        wptr, wbytes, stream), "fused_orthocache_attention")

    meta: Dict[str, Any] = {}
    if return_mask:
        meta["eviction_mask"] = mask
    return out, _finish_meta(meta, ws, num_tiles, stats)
