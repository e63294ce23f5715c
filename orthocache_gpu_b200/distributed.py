"""Sequence-sharded decode: one long sequence split over GPUs.

For contexts too long for one GPU (or to cut the latency of one decode
step), every rank holds a contiguous, tile-aligned range of the sequence's
K / V.  Each rank runs the fused Cauchy-Schwarz-gated decode over its range
and keeps the merged softmax state per query head — the running max m (log2
units), the probability sum l and the unnormalised accumulator acc — instead
of the normalised output.  One all-gather (NCCL over NVLink, a few KB per
rank) exchanges the states and every rank merges them with the library's
log-sum-exp merge, so all ranks end with the output of the whole sequence.

The gate is per tile, so sharding on tile boundaries gives exactly the
tiles (and the eviction decisions) of the unsharded call; only the
floating-point summation order of the merge differs.  A rank whose tiles are
all evicted contributes m = -1e9, l = 0 (zero weight).

The reference has no multi-GPU path; its single-GPU counterpart is
``fused_orthocache_attention_v3_gqa`` (gqa_eviction.py:511-639), and the
merge restates its split-K reduction (gqa_eviction.py:430-495) across ranks.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .fwht_fused_prototype import TILE_SIZE


def shard_range(seq_len: int, world_size: int, rank: int, tile_size: int = TILE_SIZE) -> Tuple[int, int]:
    """Token range [start, stop) of ``rank``: near-equal whole-tile shards in rank order."""
    assert seq_len % tile_size == 0, f"seq_len {seq_len} not divisible by tile_size {tile_size}"
    assert 0 <= rank < world_size
    tiles = seq_len // tile_size
    lo = rank * tiles // world_size
    hi = (rank + 1) * tiles // world_size
    return lo * tile_size, hi * tile_size


def shard_partials(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, tau: float,
                   num_query_groups: int, num_splits: Optional[int] = None,
                   k_scale: float = 1.0, stats: bool = True,
                   seq_len_dev: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """This rank's merged state over its K / V shard.

    q (Hq, hd); keys / values (KVH, S_shard, hd).  Returns float32 tensors
    m (Hq,), l (Hq,), acc (Hq, hd) and the number of retained tiles (-1 with
    ``stats=False``, which skips that host synchronisation).  ``seq_len_dev``
    (one int32 on the device, a multiple of 64): decode only that many leading
    tokens of keys / values, read by the kernel (CUDA-graph friendly).
    """
    num_kv_heads, seq_len, head_dim = keys.shape
    G = num_query_groups
    assert q.shape[0] == num_kv_heads * G, (
        f"num_query_heads ({q.shape[0]}) != num_kv_heads ({num_kv_heads}) × G ({G})")
    assert seq_len % TILE_SIZE == 0, f"seq_len {seq_len} not divisible by tile_size {TILE_SIZE}"
    if k_scale != 1.0:
        q = q * k_scale
    dev = _lib.require_cuda(q, keys, values)
    num_tiles = seq_len // TILE_SIZE
    lib = _lib.load()
    if num_splits is None:
        num_splits = lib.oc_auto_num_splits(num_tiles, _lib.num_sms(dev))
    num_splits = max(1, min(num_splits, max(num_tiles, 1)))
    q = q if q.stride(-1) == 1 else q.contiguous()
    keys, values = _lib.harmonize_kv(keys, values)
    keys, values = _lib.prepare_kv(keys), _lib.prepare_kv(values)
    hq = q.shape[0]
    m = torch.empty(hq, dtype=torch.float32, device=dev)
    l = torch.empty(hq, dtype=torch.float32, device=dev)
    acc = torch.empty((hq, head_dim), dtype=torch.float32, device=dev)
    stream = _lib.stream_ptr(dev)
    ws = _lib.workspace(dev, stream)
    wptr, wbytes = ws.get(_lib.workspace_bytes(num_kv_heads, G, num_tiles, head_dim))
    _lib.check(lib.oc_fused_attention_v3_shard(
        q.data_ptr(), _lib.dtype_code(q), q.stride(0),
        keys.data_ptr(), _lib.dtype_code(keys), keys.stride(0), keys.stride(1),
        values.data_ptr(), _lib.dtype_code(values), values.stride(0), values.stride(1),
        num_kv_heads, G, seq_len, head_dim, float(tau), num_splits, _lib.num_sms(dev),
        m.data_ptr(), l.data_ptr(), acc.data_ptr(), 0, _lib.ptr(seq_len_dev), ws.retained_ptr if stats else 0,
        ws.status_ptr,
        wptr, wbytes, stream), "oc_fused_attention_v3_shard")
    return m, l, acc, (_lib.read_stats(ws) if stats else -1)


def pack_state(m: torch.Tensor, l: torch.Tensor, acc: torch.Tensor) -> torch.Tensor:
    """One contiguous float32 row per query head: [m, l, acc...] (Hq, hd + 2)."""
    return torch.cat([m[:, None], l[:, None], acc], dim=1).contiguous()


def gather_states(packed: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather the packed states of every rank: (world, Hq, hd + 2).

    One collective per decode step; NCCL gathers into one tensor, other
    backends (gloo, for host-side tests) through a list.
    """
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(packed.shape), dtype=packed.dtype, device=packed.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, packed, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), packed, group=group)
    return out


def unpack_for_merge(gathered: torch.Tensor):
    """(world, Hq, hd+2) -> m (Hq, world), l (Hq, world), acc (Hq, world, hd), contiguous."""
    g = gathered.permute(1, 0, 2)
    return g[..., 0].contiguous(), g[..., 1].contiguous(), g[..., 2:].contiguous()


def merge_states(m: torch.Tensor, l: torch.Tensor, acc: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """Log-sum-exp merge on the GPU (oc_lse_merge): m, l (Hq, P) log2 units; acc (Hq, P, hd)."""
    dev = _lib.require_cuda(m, l, acc)
    hq, parts, hd = acc.shape
    out = torch.empty((hq, hd), dtype=out_dtype, device=dev)
    _lib.check(_lib.load().oc_lse_merge(m.data_ptr(), l.data_ptr(), acc.data_ptr(), hq, parts, hd,
                                        out.data_ptr(), _lib.dtype_code(out), _lib.stream_ptr(dev)),
               "oc_lse_merge")
    return out


def sequence_sharded_decode(q: torch.Tensor, keys_shard: torch.Tensor, values_shard: torch.Tensor, tau: float,
                            num_query_groups: int, group=None, num_splits: Optional[int] = None,
                            k_scale: float = 1.0):
    """Decode one sequence whose K / V are sharded over the ranks of ``group``.

    Every rank passes the same q (Hq, hd) and its own tile-aligned shard
    (``shard_range``) of keys / values (KVH, S_shard, hd).  Returns the
    output (Hq, hd) in q's dtype on every rank, and metadata.  Nothing is read
    back to the host before the all-gather; a device error of this rank's
    launch stays in the stream's status word (``check_status()``).
    """
    input_dtype = q.dtype
    # no host synchronisation before the collective: the retained count is not read
    # (the sticky status word stays checkable with check_status())
    m, l, acc, kept = shard_partials(q, keys_shard, values_shard, tau, num_query_groups, num_splits, k_scale,
                                     stats=False)
    gathered = gather_states(pack_state(m, l, acc), group)
    mm, ll, aa = unpack_for_merge(gathered)
    out = merge_states(mm, ll, aa, input_dtype)
    meta = {"layout": "sequence_sharded", "world_size": gathered.shape[0],
            "shard_tiles": keys_shard.shape[1] // TILE_SIZE,
            "gate_type": "cauchy_schwarz", "num_query_groups": num_query_groups}
    return out, meta
