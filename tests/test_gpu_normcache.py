"""GPU parity of the spectral norm cache, the O(1) decode gate and the cached-gate decode.

Against the reference-generated golden vectors (``norm_cache``, ``decode_gate``
cases of tests/golden) and the CPU oracle: norms within 1e-5 relative (the
float32 summation order differs), gate masks bit-exact except tiles whose
bound lies within 1e-5 relative of tau * 64 * head_dim, outputs within 1e-5
(float32) / 2e-3 (float16, bfloat16) max-abs.
"""

import numpy as np
import pytest
import torch

import orthocache_gpu_b200 as oc
from cases import case_inputs
from helpers import as_np, assert_close, assert_mask, cast_np, golden
from oracle import orthocache_oracle as orc
from orthocache_gpu_b200.synthetic import gqa_inputs, tile_mixture

pytestmark = pytest.mark.gpu
DEV = "cuda"
QH_ATOL = 4e-3  # |q_high| of a query without high band: sqrt of float32 rounding noise


def _mid_tau(q, norms, G, hd):
    """A tau between two neighbouring per-tile bounds near their median (no tile near the threshold)."""
    b = np.sort(np.concatenate([orc.decode_gate(qq, nn, 1.0, nn.shape[-1], G)[2].ravel()
                                for qq, nn in zip(q.reshape(-1, *q.shape[-2:]), norms.reshape(-1, *norms.shape[-2:]))]))
    i = len(b) // 2
    while i + 1 < len(b) and b[i + 1] - b[i] < 1e-3 * b[i]:
        i += 1
    return float((b[i] + b[i + 1]) / 2) / (64 * hd)


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to(DEV)


def test_norm_cache_matches_reference_golden():
    inp, z = case_inputs("norm_cache"), golden("norm_cache")
    w = oc.generate_walsh_matrix(64)
    for i, hs in enumerate(z["thresholds"]):
        c = oc.SpectralNormCache(4, 16, DEV).populate_from_keys(T(inp["keys"]), w, high_start=int(hs), high_end=64)
        np.testing.assert_allclose(as_np(c.cache), z[f"norms_{i}"], rtol=1e-5, atol=0)
        assert c.is_populated and (as_np(c.valid_tiles) == z[f"valid_{i}"]).all()


@pytest.mark.parametrize("hd", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
def test_tile_high_norms_head_dims_and_dtypes(hd, dt):
    rng = np.random.default_rng(hd)
    keys, _ = tile_mixture(rng, (3,), 10, hd)
    for band in ((48, 64), (32, 64), (1, 8), (0, 64)):
        got = as_np(oc.tile_high_norms(T(keys, dt), *band))
        ref = orc.tile_high_norms(cast_np(keys, dt), *band)
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_norm_cache_update_and_append_follow_the_reference_semantics():
    rng = np.random.default_rng(3)
    keys, _ = tile_mixture(rng, (2,), 6, 64)
    w = oc.generate_walsh_matrix(64)
    c = oc.SpectralNormCache(2, 8, DEV)
    assert not c.is_populated
    c.update_prefill(1, 2, T(keys[1, 128:192]), w, 48, 64)
    assert c.valid_tiles.tolist() == [0, 3]
    np.testing.assert_allclose(c.get_norm(1, 2), orc.tile_high_norms(keys[1, 128:192])[0], rtol=1e-5)
    c.populate_from_keys(T(keys[:, :256]), w)             # 4 tiles of both heads
    c.append_tiles(T(keys[:, 256:]), 4)                     # tiles 4, 5
    np.testing.assert_allclose(as_np(c.cache)[:, :6], orc.tile_high_norms(keys), rtol=1e-5)
    assert c.valid_tiles.tolist() == [6, 6] and c.get_norms_batch(0).numel() == 6
    assert c.memory_bytes == 2 * 8 * 4 and "2 heads" in c.summary()


@pytest.mark.parametrize("tight", [True, False])
def test_decode_gate_matches_reference_golden(tight):
    inp, z = case_inputs("decode_gate"), golden("decode_gate")
    q, nrm = T(inp["q"]), T(inp["norms"])
    np.testing.assert_allclose(as_np(oc.compute_q_high_norm_exact(q)), z["q_high"], rtol=1e-5, atol=QH_ATOL)
    for i, tau in enumerate(z["thresholds"]):
        evict, qn = oc.decode_gate(q, nrm, tau, 12, 4, tight=tight)
        assert evict.dtype == torch.bool and evict.shape == (4, 16)
        np.testing.assert_allclose(as_np(qn), z[f"qn_{i}_{int(tight)}"], rtol=1e-5, atol=QH_ATOL)
        _, _, bound = orc.decode_gate(inp["q"], inp["norms"], tau, 12, 4, tight=tight)
        assert_mask(evict, z[f"evict_{i}_{int(tight)}"], bound, tau * 64 * 64, f"gate tau={tau} tight={tight}")


@pytest.mark.parametrize("q_stat", ["max", "median"])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_cached_decode_against_oracle(q_stat, dt):
    x = gqa_inputs(2, 4, 2048, 128, seed=7, batch=3)
    q, k, v = (cast_np(a, dt) for a in (x.q, x.keys, x.values))
    norms = orc.tile_high_norms(k)                            # (3, 2, 32), band [48, 64)
    tau = _mid_tau(q, norms, 4, 128)                          # about half the tiles evicted
    out, meta = oc.fused_orthocache_attention_cached(T(x.q, dt), T(x.keys, dt), T(x.values, dt), T(norms), tau, 4,
                                                     q_stat=q_stat, return_mask=True)
    kept = 0
    for b in range(3):
        ref, ev, bound = orc.cached_attention(q[b], k[b], v[b], norms[b], tau, 4, stat=q_stat)
        assert_mask(~as_np(meta["evict_mask"][b]).astype(bool), ~ev, bound, tau * 64 * 128, f"cached seq {b}")
        near = orc.near_threshold(bound, tau * 64 * 128)
        if near.any():
            ref, ev, _ = orc.cached_attention(q[b], k[b], v[b], norms[b], tau, 4, stat=q_stat,
                                              forced=(near, as_np(meta["evict_mask"][b]).astype(bool)))
        kept += int((~ev).sum())
        assert_close(out[b], ref, dt, f"cached seq {b} {q_stat}")
    assert meta["tiles_retained"] == kept and 0.1 < meta["eviction_rate"] < 0.9


def test_cached_decode_never_reads_evicted_tiles():
    # poison K and V of every evicted tile with NaN: a kernel that read them
    # would produce NaN; the output must equal the oracle on the clean data
    x = gqa_inputs(2, 4, 4096, 128, seed=11)
    dt = torch.bfloat16
    q, k, v = (cast_np(a, dt) for a in (x.q, x.keys, x.values))
    norms = orc.tile_high_norms(k)
    tau = _mid_tau(q, norms, 4, 128)
    ref, ev, bound = orc.cached_attention(q, k, v, norms, tau, 4)
    assert ev.any() and not ev.all() and not orc.near_threshold(bound, tau * 64 * 128).any()
    kd, vd = T(x.keys, dt), T(x.values, dt)
    for h in range(2):
        for t in np.flatnonzero(ev[h]):
            kd[h, 64 * t: 64 * t + 64] = float("nan")
            vd[h, 64 * t: 64 * t + 64] = float("nan")
    out, meta = oc.fused_orthocache_attention_cached(T(x.q, dt), kd, vd, T(norms), tau, 4)
    assert torch.isfinite(out).all()
    assert_close(out, ref, dt, "cached decode with poisoned evicted tiles")
    assert meta["tiles_evicted"] == int(ev.sum())


def test_cached_decode_all_evicted_and_none_evicted():
    x = gqa_inputs(2, 2, 1024, 64, seed=12)
    q, k, v = T(x.q), T(x.keys), T(x.values)
    norms = oc.tile_high_norms(k)
    out, meta = oc.fused_orthocache_attention_cached(q, k, v, norms, 1e30, 2)
    assert meta["tiles_retained"] == 0 and out.abs().max().item() == 0.0
    out, meta = oc.fused_orthocache_attention_cached(q, k, v, norms, -1.0, 2)
    assert meta["tiles_evicted"] == 0
    ref, _ = orc.v3_gqa_attention(x.q, x.keys, x.values, -1.0, 2)
    assert_close(out, ref, torch.float32, "cached decode, nothing evicted")


def test_cached_decode_with_a_norm_cache_object_and_longer_capacity():
    # the cache holds more tiles than the keys: only the first S/64 are used
    x = gqa_inputs(2, 4, 1024, 128, seed=13)
    dt = torch.float16
    k = T(x.keys, dt)
    c = oc.SpectralNormCache(2, 64, DEV).populate_from_keys(k, oc.generate_walsh_matrix(64))
    nrm = as_np(c.cache)[:, :16]
    tau = _mid_tau(cast_np(x.q, dt), nrm, 4, 128)
    out, meta = oc.fused_orthocache_attention_cached(T(x.q, dt), k, T(x.values, dt), c, tau, 4, return_mask=True)
    ref, ev, bound = orc.cached_attention(cast_np(x.q, dt), cast_np(x.keys, dt), cast_np(x.values, dt), nrm, tau, 4,
                                          forced=(orc.near_threshold(orc.decode_gate(cast_np(x.q, dt), nrm, tau, 16,
                                                                                      4)[2], tau * 64 * 128),
                                                  as_np(meta["evict_mask"]).astype(bool)))
    assert_close(out, ref, dt, "cached decode from a SpectralNormCache")
