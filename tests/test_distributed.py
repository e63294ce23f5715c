"""Sequence-sharded decode (one long sequence over several ranks).

CPU: world_size-2 gloo ranks check the host side — tile-aligned shard
ranges, packing, the all-gather layout and the merge — with partial states
computed by the NumPy oracle, against the oracle's unsharded V3 output.
GPU: the CUDA shard kernel and the CUDA log-sum-exp merge, with the ranks
emulated on one GPU (and over NCCL when two GPUs are visible).
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import orthocache_oracle as orc
from orthocache_gpu_b200 import distributed as ocd
from orthocache_gpu_b200.synthetic import gqa_inputs

from helpers import TOL

KVH, G, HD, SEQ, TAU = 2, 4, 64, 64 * 24, 150.0


def _inputs():
    return gqa_inputs(KVH, G, SEQ, HD, seed=21)


def _oracle_partial(q, keys, values, tau):
    """Merged softmax state (natural-log units) of one shard: m, l (Hq,), acc (Hq, hd)."""
    qg = q.astype(np.float64).reshape(KVH, G, HD)
    keep = orc.cs_keep(orc.cs_bound(qg, keys), tau)          # (KVH, T)
    hq = KVH * G
    m = np.full(hq, -1e9)
    l = np.zeros(hq)
    acc = np.zeros((hq, HD))
    for h in range(KVH):
        rows = np.repeat(keep[h], 64)
        if not rows.any():
            continue
        k = keys[h][rows].astype(np.float64)
        v = values[h][rows].astype(np.float64)
        for i in range(G):
            s = k @ qg[h, i] / np.sqrt(HD)
            mx = s.max()
            p = np.exp(s - mx)
            m[h * G + i], l[h * G + i], acc[h * G + i] = mx, p.sum(), p @ v
    return m, l, acc


def test_shard_ranges_cover_the_sequence_in_whole_tiles():
    for world in (1, 2, 3, 8):
        spans = [ocd.shard_range(64 * 37, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 64 * 37
        for (a, b), (c, _) in zip(spans, spans[1:]):
            assert b == c
        assert all((b - a) % 64 == 0 and b - a >= 64 * (37 // world) for a, b in spans)


def test_empty_shard_merges_with_zero_weight():
    m, l, acc = np.array([[0.5, -1e9]]), np.array([[2.0, 0.0]]), np.array([[[1.0, 2.0], [0.0, 0.0]]])
    np.testing.assert_allclose(orc.lse_merge(m, l, acc), [[0.5, 1.0]])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        inp = _inputs()
        a, b = ocd.shard_range(SEQ, world, rank)
        m, l, acc = _oracle_partial(inp.q, inp.keys[:, a:b], inp.values[:, a:b], TAU)
        packed = ocd.pack_state(*(torch.from_numpy(x).float() for x in (m, l, acc)))
        gathered = ocd.gather_states(packed)
        mm, ll, aa = ocd.unpack_for_merge(gathered)
        out = orc.lse_merge(mm.double().numpy(), ll.double().numpy(), aa.double().numpy())
        result[rank] = torch.from_numpy(out)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_match_the_unsharded_oracle():
    world = 2
    result = mp.Manager().dict()
    mp.spawn(_gloo_rank, args=(world, _free_port(), result), nprocs=world, join=True)
    inp = _inputs()
    ref, _ = orc.v3_gqa_attention(inp.q, inp.keys, inp.values, TAU, G)
    for r in range(world):
        np.testing.assert_allclose(result[r].numpy(), ref, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 3])
def test_gpu_shards_merged_on_one_gpu_match_v3(world):
    import orthocache_gpu_b200 as oc
    inp = _inputs()
    q, k, v = inp.torch(torch.bfloat16, "cuda")
    ref32, _ = orc.v3_gqa_attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), TAU, G)
    states = []
    for r in range(world):
        a, b = ocd.shard_range(SEQ, world, r)
        m, l, acc, _ = ocd.shard_partials(q, k[:, a:b], v[:, a:b], TAU, G)
        states.append(ocd.pack_state(m, l, acc))
    mm, ll, aa = ocd.unpack_for_merge(torch.stack(states))
    out = ocd.merge_states(mm, ll, aa, q.dtype)
    full, _ = oc.fused_orthocache_attention_v3_gqa(q, k, v, TAU, G)
    assert (out.float().cpu().numpy() - ref32).__abs__().max() <= TOL[torch.bfloat16]
    assert (out.float() - full.float()).abs().max().item() <= TOL[torch.bfloat16]


def _nccl_rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        inp = _inputs()
        q, k, v = inp.torch(torch.bfloat16, f"cuda:{rank}")
        a, b = ocd.shard_range(SEQ, world, rank)
        out, meta = ocd.sequence_sharded_decode(q, k[:, a:b].contiguous(), v[:, a:b].contiguous(), TAU, G)
        result[rank] = out.float().cpu()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_two_ranks_match_the_unsharded_oracle():
    world = 2
    result = mp.Manager().dict()
    mp.spawn(_nccl_rank, args=(world, _free_port(), result), nprocs=world, join=True)
    inp = _inputs()
    q, k, v = inp.torch(torch.bfloat16, "cpu")
    ref, _ = orc.v3_gqa_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), TAU, G)
    for r in range(world):
        assert np.abs(result[r].numpy() - ref).max() <= TOL[torch.bfloat16]
