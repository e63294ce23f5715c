"""GPU parity at the full sizes of the benchmarked configurations.

Every configuration the benchmark times is checked here at its own size
against the CPU oracle on seeded inputs: masks bit-exact except tiles whose
score lies within 1e-5 relative of the threshold (those tiles take the GPU's
decision in the oracle, so outputs and retained counts are compared in every
case); outputs within 2e-3 max-abs (float16 / bfloat16).

* V2: 32 heads x 8K / 16K / 32K tokens, head_dim 128, float16, ζ_max 5.0 and 1.0;
* V3: batch 16 x 8 kv heads (G = 4) x 32K, bfloat16, half of the query
  heads high-band-zeroed, τ 1.0 and 150;
* paged GQA: 64 sequences of U[2K, 64K] tokens (multiples of 64), 16-token
  pages in a permuted pool, 32 / 8 heads, float16, τ 1.0 and 150;
* one 512K-token sequence, 8 kv heads with G = 8, bfloat16, decoded in 2, 4
  and 8 tile-aligned shards (the shard kernel + the log-sum-exp merge, as the
  multi-GPU path runs them) against the unsharded oracle.

Inputs are generated per head / sequence on the host so that the oracle's
float32 copies stay a few hundred MB at a time.
"""

import numpy as np
import pytest
import torch

import orthocache_gpu_b200 as oc
from helpers import as_np, assert_close, assert_mask, gpu_forced
from oracle import orthocache_oracle as orc
from orthocache_gpu_b200 import distributed as ocd
from orthocache_gpu_b200.synthetic import tile_mixture, zero_high_band_queries

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rt(a, dt):
    """float32 numpy array rounded through a torch dtype."""
    return torch.from_numpy(np.ascontiguousarray(a)).to(dt).float().numpy()


def _heads(seed, n, seq, hd, dt):
    """Per-head seeded K / V (each (seq, hd)) rounded through dt, as a generator."""
    for h in range(n):
        rng = np.random.default_rng([seed, h])
        k, _ = tile_mixture(rng, (), seq // 64, hd)
        v = rng.standard_normal(k.shape, dtype=np.float32)
        yield _rt(k, dt), _rt(v, dt)


@pytest.mark.parametrize("seq", [8192, 16384, 32768])
def test_v2_config2_full_size(seq):
    H, HD, dt = 32, 128, torch.float16
    k = torch.empty((H, seq, HD), dtype=dt, device=DEV)
    v = torch.empty_like(k)
    for h, (kh, vh) in enumerate(_heads(seq, H, seq, HD, dt)):
        k[h] = torch.from_numpy(kh).to(dt)
        v[h] = torch.from_numpy(vh).to(dt)
    qn = _rt(np.random.default_rng(seq + 1).standard_normal((H, HD), dtype=np.float32), dt)
    q = torch.from_numpy(qn).to(dt).to(DEV)
    runs = {thr: oc.fused_orthocache_attention_v2(q, k, v, thr, return_mask=True) for thr in (5.0, 1.0)}
    for thr, (out, gm) in runs.items():
        mask = as_np(gm["eviction_mask"]).astype(bool)
        kept, err = 0, 0.0
        for h, (kh, vh) in enumerate(_heads(seq, H, seq, HD, dt)):
            zeta = orc.tile_zeta(kh)
            keep = orc.zeta_keep(zeta, thr)
            assert_mask(mask[h], keep, zeta, thr, f"v2 {seq} thr={thr} head {h}")
            near, gk = gpu_forced(mask[h], zeta, thr)
            keep = np.where(near, gk, keep)
            kept += int(keep.sum())
            ref = orc.masked_decode(qn[h], kh, vh, keep)
            err = max(err, float(np.abs(as_np(out[h]) - ref).max()))
        assert gm["tiles_retained"] == kept
        assert err <= 2e-3, f"v2 {seq} thr={thr}: max abs error {err:.3g}"
        if thr == 1.0:
            assert 0.4 < gm["eviction_rate"] < 0.6


def test_v3_config3_full_size():
    B, KVH, G, S, HD, dt = 16, 8, 4, 32768, 128, torch.bfloat16
    k = torch.empty((B, KVH, S, HD), dtype=dt, device=DEV)
    v = torch.empty_like(k)
    for b in range(B):
        for h, (kh, vh) in enumerate(_heads(1000 + b, KVH, S, HD, dt)):
            k[b, h] = torch.from_numpy(kh).to(dt)
            v[b, h] = torch.from_numpy(vh).to(dt)
    qn = _rt(zero_high_band_queries(np.random.default_rng(77).standard_normal((B, KVH * G, HD), dtype=np.float32)), dt)
    q = torch.from_numpy(qn).to(dt).to(DEV)
    runs = {tau: oc.fused_orthocache_attention_v3_gqa(q, k, v, tau, G, return_mask=True) for tau in (1.0, 150.0)}
    outs = {tau: as_np(o) for tau, (o, _) in runs.items()}
    masks = {tau: as_np(m["eviction_mask"]).astype(bool) for tau, (_, m) in runs.items()}
    kept = {tau: 0 for tau in runs}
    err = {tau: 0.0 for tau in runs}
    for b in range(B):
        for h, (kh, vh) in enumerate(_heads(1000 + b, KVH, S, HD, dt)):
            qg = qn[b, h * G:(h + 1) * G]
            bound = orc.cs_bound(qg[None], kh[None])[0]
            for tau in runs:
                keep = orc.cs_keep(bound, tau)
                assert_mask(masks[tau][b, h], keep, bound, tau, f"v3 tau={tau} seq {b} head {h}")
                near, gk = gpu_forced(masks[tau][b, h], bound, tau)
                keep = np.where(near, gk, keep)
                kept[tau] += int(keep.sum())
                for g in range(G):
                    ref = orc.masked_decode(qg[g], kh, vh, keep)
                    err[tau] = max(err[tau], float(np.abs(outs[tau][b, h * G + g] - ref).max()))
    for tau, (_, gm) in runs.items():
        assert gm["tiles_retained"] == kept[tau], f"tau={tau}"
        assert err[tau] <= 2e-3, f"v3 tau={tau}: max abs error {err[tau]:.3g}"
    assert runs[1.0][1]["eviction_rate"] < 0.01 and 0.4 < runs[150.0][1]["eviction_rate"] < 0.6


def _paged_config4_lengths():
    rng = np.random.default_rng(0)
    lens = rng.integers(2048, 65536 + 1, size=64)
    return (lens - lens % 64).astype(np.int64)


def test_paged_config4_full_size():
    NS, KVH, G, HD, BS, dt = 64, 8, 4, 128, 16, torch.float16
    lens = _paged_config4_lengths()
    nblk = lens // BS
    total = int(nblk.sum())
    perm = torch.from_numpy(np.random.default_rng(1).permutation(total).astype(np.int64)).to(DEV)
    kc = torch.empty((total, KVH, BS, HD), dtype=dt, device=DEV)
    vc = torch.empty_like(kc)
    tables = torch.zeros((NS, int(nblk.max())), dtype=torch.int32, device=DEV)
    pos = 0

    def seq_heads(s):
        return list(_heads(5000 + s, KVH, int(lens[s]), HD, dt))

    for s in range(NS):
        nb = int(nblk[s])
        pages = perm[pos:pos + nb]
        pos += nb
        hs = seq_heads(s)
        ks = torch.from_numpy(np.stack([a for a, _ in hs])).to(dt).to(DEV)    # (KVH, L, HD)
        vs = torch.from_numpy(np.stack([b for _, b in hs])).to(dt).to(DEV)
        kc[pages] = ks.reshape(KVH, nb, BS, HD).permute(1, 0, 2, 3)
        vc[pages] = vs.reshape(KVH, nb, BS, HD).permute(1, 0, 2, 3)
        tables[s, :nb] = pages.to(torch.int32)
        tables[s, nb:] = pages[0].to(torch.int32)
    qn = _rt(zero_high_band_queries(np.random.default_rng(9).standard_normal((NS, KVH * G, HD), dtype=np.float32)), dt)
    q = torch.from_numpy(qn).to(dt).to(DEV)
    sl = torch.from_numpy(lens.astype(np.int32)).to(DEV)
    runs = {tau: oc.fused_orthocache_attention_paged(q, kc, vc, tables, None, tau=tau, seq_lens=sl, return_mask=True)
            for tau in (1.0, 150.0)}
    outs = {tau: as_np(o) for tau, (o, _) in runs.items()}
    masks = {tau: as_np(m["eviction_mask"]).astype(bool) for tau, (_, m) in runs.items()}
    kept = {tau: 0 for tau in runs}
    err = {tau: 0.0 for tau in runs}
    for s in range(NS):
        nt = int(lens[s]) // 64
        for tau in runs:
            assert not masks[tau][s, :, nt:].any(), "mask set beyond the sequence's length"
        for h, (kh, vh) in enumerate(seq_heads(s)):
            qg = qn[s, h * G:(h + 1) * G]
            bound = orc.cs_bound(qg[None], kh[None])[0]
            for tau in runs:
                keep = orc.cs_keep(bound, tau)
                assert_mask(masks[tau][s, h, :nt], keep, bound, tau, f"paged tau={tau} seq {s} head {h}")
                near, gk = gpu_forced(masks[tau][s, h, :nt], bound, tau)
                keep = np.where(near, gk, keep)
                kept[tau] += int(keep.sum())
                for g in range(G):
                    ref = orc.masked_decode(qg[g], kh, vh, keep)
                    err[tau] = max(err[tau], float(np.abs(outs[tau][s, h * G + g] - ref).max()))
    for tau, (_, gm) in runs.items():
        assert gm["tiles_retained"] == kept[tau], f"tau={tau}"
        assert err[tau] <= 2e-3, f"paged tau={tau}: max abs error {err[tau]:.3g}"


def test_long_context_512k_sharded_decode():
    KVH, G, S, HD, dt, tau = 8, 8, 512 * 1024, 128, torch.bfloat16, 150.0
    k = torch.empty((KVH, S, HD), dtype=dt, device=DEV)
    v = torch.empty_like(k)
    for h, (kh, vh) in enumerate(_heads(512, KVH, S, HD, dt)):
        k[h] = torch.from_numpy(kh).to(dt)
        v[h] = torch.from_numpy(vh).to(dt)
    qn = _rt(zero_high_band_queries(np.random.default_rng(512).standard_normal((KVH * G, HD), dtype=np.float32)), dt)
    q = torch.from_numpy(qn).to(dt).to(DEV)
    full, gm = oc.fused_orthocache_attention_v3_gqa(q, k, v, tau, G, return_mask=True)
    mask = as_np(gm["eviction_mask"]).astype(bool)
    sharded = {}
    for world in (2, 4, 8):
        ms, ls, accs = [], [], []
        for r in range(world):
            a, b = ocd.shard_range(S, world, r)
            m, l, acc, _ = ocd.shard_partials(q, k[:, a:b], v[:, a:b], tau, G, stats=False)
            ms.append(m)
            ls.append(l)
            accs.append(acc)
        sharded[world] = as_np(ocd.merge_states(torch.stack(ms, 1).contiguous(), torch.stack(ls, 1).contiguous(),
                                                torch.stack(accs, 1).contiguous(), dt))
    oc.check_status()
    out = as_np(full)
    kept, err = 0, {w: 0.0 for w in [1, *sharded]}
    for h, (kh, vh) in enumerate(_heads(512, KVH, S, HD, dt)):
        qg = qn[h * G:(h + 1) * G]
        bound = orc.cs_bound(qg[None], kh[None])[0]
        keep = orc.cs_keep(bound, tau)
        assert_mask(mask[h], keep, bound, tau, f"512K head {h}")
        near, gk = gpu_forced(mask[h], bound, tau)
        keep = np.where(near, gk, keep)
        kept += int(keep.sum())
        for g in range(G):
            ref = orc.masked_decode(qg[g], kh, vh, keep)
            err[1] = max(err[1], float(np.abs(out[h * G + g] - ref).max()))
            for w, o in sharded.items():
                err[w] = max(err[w], float(np.abs(o[h * G + g] - ref).max()))
    assert gm["tiles_retained"] == kept
    assert 0.4 < gm["eviction_rate"] < 0.6
    for w, e in err.items():
        assert e <= 2e-3, f"512K, {w} shard(s): max abs error {e:.3g}"


def test_cached_gate_decode_config3_full_size():
    # the O(1) cached-norm gate at the V3 shapes: norms scored once on the GPU
    # (band [48, 64)), tau between two neighbouring bounds at the median
    B, KVH, G, S, HD, dt = 16, 8, 4, 32768, 128, torch.bfloat16
    k = torch.empty((B, KVH, S, HD), dtype=dt, device=DEV)
    v = torch.empty_like(k)
    for b in range(B):
        for h, (kh, vh) in enumerate(_heads(3000 + b, KVH, S, HD, dt)):
            k[b, h] = torch.from_numpy(kh).to(dt)
            v[b, h] = torch.from_numpy(vh).to(dt)
    qn = _rt(zero_high_band_queries(np.random.default_rng(78).standard_normal((B, KVH * G, HD), dtype=np.float32)), dt)
    q = torch.from_numpy(qn).to(dt).to(DEV)
    norms = oc.tile_high_norms(k.reshape(B * KVH, S, HD)).reshape(B, KVH, S // 64)
    nrm = as_np(norms)
    bounds = np.sort(np.concatenate([orc.decode_gate(qn[b], nrm[b], 1.0, S // 64, G)[2].ravel() for b in range(B)]))
    i = len(bounds) // 2
    while bounds[i + 1] - bounds[i] < 1e-3 * bounds[i]:
        i += 1
    tau = float((bounds[i] + bounds[i + 1]) / 2) / (64 * HD)
    out, meta = oc.fused_orthocache_attention_cached(q, k, v, norms, tau, G, return_mask=True)
    out = as_np(out)
    ev_gpu = as_np(meta["evict_mask"]).astype(bool)
    kept, err = 0, 0.0
    for b in range(B):
        heads = list(_heads(3000 + b, KVH, S, HD, dt))
        kh = np.stack([a for a, _ in heads])
        np.testing.assert_allclose(nrm[b], orc.tile_high_norms(kh), rtol=1e-5)
        ref, ev, bound = orc.cached_attention(qn[b], kh, np.stack([c for _, c in heads]), nrm[b], tau, G)
        assert_mask(~ev_gpu[b], ~ev, bound, tau * 64 * HD, f"cached seq {b}")
        kept += int((~ev).sum())
        err = max(err, float(np.abs(out[b] - ref).max()))
    assert meta["tiles_retained"] == kept and 0.4 < meta["eviction_rate"] < 0.6
    assert err <= 2e-3, f"cached decode: max abs error {err:.3g}"
