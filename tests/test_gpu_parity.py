"""GPU parity of the CUDA path against the reference's golden vectors and the oracle.

Masks must be bit-exact except tiles whose score lies within 1e-5 relative of
the threshold (listed, not failed); outputs within 1e-5 (float32) or 2e-3
(float16 / bfloat16) max-abs.  All calls go through the public API, which
calls the C ABI of liborthocache_b200.so.
"""

import numpy as np
import pytest
import torch

import orthocache_gpu_b200 as oc
from cases import case_inputs, fp8_quantize
from helpers import as_np, assert_close, assert_mask, cast_np, golden, gpu_forced
from oracle import orthocache_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to(DEV)


# ------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("name", ["mask_semantic", "mask_random", "mask_mixture_hd64"])
def test_mask_kernel_matches_reference_golden(name):
    inp, z = case_inputs(name), golden(name)
    for i, thr in enumerate(z["thresholds"]):
        mask, zeta = oc.triton_fwht_eviction(T(inp["keys"]), thr, return_zeta=True)
        assert mask.dtype == torch.bool and zeta.dtype == torch.float32
        np.testing.assert_allclose(as_np(zeta), z[f"zeta_{i}"], rtol=1e-4, atol=1e-6)
        assert_mask(mask, z[f"mask_{i}"], z[f"zeta_{i}"], thr, name)


def test_mask_kernel_bf16_and_fp16_keys():
    inp = case_inputs("mask_random")
    for dt in (torch.float16, torch.bfloat16):
        k = cast_np(inp["keys"], dt)
        zref = orc.tile_zeta(k)
        mask, zeta = oc.triton_fwht_eviction(T(inp["keys"], dt), 4.5, return_zeta=True)
        np.testing.assert_allclose(as_np(zeta), zref, rtol=1e-4)
        assert_mask(mask, orc.zeta_mask(zref, 4.5), zref, 4.5, str(dt))


def test_v1_config1_matches_reference_golden():
    inp, z = case_inputs("v1_config1"), golden("v1_config1")
    zeta = orc.tile_zeta(inp["keys"])
    for i, thr in enumerate(z["thresholds"]):
        out, meta = oc.fused_orthocache_attention(T(inp["q"]), T(inp["keys"]), T(inp["values"]), thr,
                                                  return_mask=True)
        assert out.shape == (1, 128) and out.dtype == torch.float32
        near = assert_mask(meta["eviction_mask"], z[f"mask_{i}"], zeta, thr, "v1")
        if len(near) == 0:  # the reference's own output applies
            assert meta["tiles_retained"] == int(z[f"retained_{i}"])
            assert_close(out, z[f"out_{i}"], torch.float32, f"v1 thr={thr}")
        else:  # the oracle with the GPU's decisions on the listed tiles
            ref, rm = orc.v1_attention(inp["q"], inp["keys"], inp["values"], thr,
                                       forced=gpu_forced(meta["eviction_mask"], zeta, thr))
            assert meta["tiles_retained"] == rm["tiles_retained"]
            assert_close(out, ref, torch.float32, f"v1 thr={thr} (near tiles forced)")


@pytest.mark.parametrize("name", ["v2_f16", "v2_bf16_hd64"])
def test_v2_matches_reference_golden(name):
    inp, z = case_inputs(name), golden(name)
    dt = getattr(torch, inp["dtype"])
    for i, thr in enumerate(z["thresholds"]):
        for splits in (None, 1, 3):
            out, meta = oc.fused_orthocache_attention_v2(T(inp["q"], dt), T(inp["keys"], dt),
                                                         T(inp["values"], dt), thr, num_splits=splits)
            assert out.dtype == dt and meta["tile_assignment"] == "interleaved"
            assert meta["tiles_retained"] == int(z[f"retained_{i}"])
            assert_close(out, z[f"out32_{i}"], dt, f"{name} thr={thr} splits={splits}")


@pytest.mark.parametrize("name", ["v3_bf16", "v3_f32_g1"])
def test_v3_matches_reference_golden(name):
    inp, z = case_inputs(name), golden(name)
    dt = getattr(torch, inp["dtype"])
    for i, tau in enumerate(z["thresholds"]):
        out, meta = oc.fused_orthocache_attention_v3_gqa(T(inp["q"], dt), T(inp["keys"], dt),
                                                         T(inp["values"], dt), tau, inp["group"])
        assert meta["gate_type"] == "cauchy_schwarz"
        assert meta["tiles_retained"] == int(z[f"retained_{i}"])
        assert meta["tiles_evicted"] == int(z[f"evicted_{i}"])
        assert_close(out, z[f"out32_{i}"], dt, f"{name} tau={tau}")


def test_paged_matches_reference_golden():
    inp, z = case_inputs("paged_f32"), golden("paged_f32")
    for i, thr in enumerate(z["thresholds"]):
        out, meta = oc.fused_orthocache_attention_paged(
            T(inp["q"]), T(inp["k_cache"]), T(inp["v_cache"]),
            torch.from_numpy(inp["block_tables"]).to(DEV), thr)
        assert meta["layout"] == "paged"
        assert_close(out, z[f"out_{i}"], torch.float32, f"paged thr={thr}")


def test_fp8_keys_match_reference_golden():
    inp, z = case_inputs("v2_fp8"), golden("v2_fp8")
    k8, scale = fp8_quantize(inp["keys"])
    for i, thr in enumerate(z["thresholds"]):
        out, _ = oc.fused_orthocache_attention_v2(T(inp["q"]), k8.to(DEV), T(inp["values"]), thr, k_scale=scale)
        assert_close(out, z[f"out_{i}"], torch.float32, f"fp8 thr={thr}")


# ------------------------------------------------------------ oracle, larger shapes
def _v2_case(h, s, hd, dt, thr, seed, splits=None):
    from orthocache_gpu_b200.synthetic import mha_inputs
    x = mha_inputs(h, s, hd, seed=seed)
    q, k, v = (cast_np(a, dt) for a in (x.q, x.keys, x.values))
    ref, meta = orc.v2_attention(q, k, v, thr)
    out, gm = oc.fused_orthocache_attention_v2(T(x.q, dt), T(x.keys, dt), T(x.values, dt), thr,
                                               num_splits=splits, return_mask=True)
    near = assert_mask(gm["eviction_mask"], meta["eviction_mask"], meta["zeta"], thr, "v2 mask")
    if len(near):
        ref, meta = orc.v2_attention(q, k, v, thr, forced=gpu_forced(gm["eviction_mask"], meta["zeta"], thr))
    assert gm["tiles_retained"] == meta["tiles_retained"]
    assert_close(out, ref, dt, f"v2 h={h} s={s} hd={hd} {dt}")
    return gm


@pytest.mark.parametrize("hd", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
def test_v2_head_dims_and_dtypes(hd, dt):
    if dt == torch.float32 and hd > 128:
        pytest.skip("float32 keys support head_dim <= 128")
    _v2_case(3, 640, hd, dt, 1.0, seed=hd)


@pytest.mark.parametrize("seq", [64, 1024, 4096])
def test_v2_config2_shapes(seq):
    gm = _v2_case(32, seq, 128, torch.float16, 1.0, seed=seq)
    assert 0.3 < gm["eviction_rate"] < 0.7


def test_v2_config2_literal_threshold():
    _v2_case(32, 2048, 128, torch.float16, 5.0, seed=5)


@pytest.mark.parametrize("splits", [1, 2, 7, 16, 64])
def test_v2_split_invariance(splits):
    _v2_case(4, 4096, 128, torch.float16, 1.0, seed=9, splits=splits)


def test_v2_no_eviction_equals_dense_and_all_evicted_is_zero():
    from orthocache_gpu_b200.synthetic import mha_inputs
    x = mha_inputs(4, 1024, 64, seed=3)
    q, k, v = T(x.q), T(x.keys), T(x.values)
    out, meta = oc.fused_orthocache_attention_v2(q, k, v, 1e6)
    assert meta["tiles_evicted"] == 0
    dense = torch.softmax((q[:, None, :] @ k.transpose(1, 2)) / 8.0, -1) @ v
    assert (out - dense[:, 0]).abs().max().item() < 1e-5
    out0, meta0 = oc.fused_orthocache_attention_v2(q, k, v, -1.0)
    assert meta0["tiles_retained"] == 0
    assert torch.isfinite(out0).all() and out0.abs().max().item() == 0.0


def test_v2_large_logits_are_finite():
    from orthocache_gpu_b200.synthetic import mha_inputs
    x = mha_inputs(2, 512, 128, seed=4)
    q = T(x.q) * 100.0
    out, _ = oc.fused_orthocache_attention_v2(q, T(x.keys), T(x.values), 1e9)
    ref, _ = orc.v2_attention(as_np(q), x.keys, x.values, 1e9)
    assert torch.isfinite(out).all()
    # logits ~1e3: float32 rounding of the logits alone is ~1e-4 relative
    np.testing.assert_allclose(as_np(out), ref, rtol=2e-3, atol=2e-3)


def test_v2_strided_pipeline_layout_is_read_in_place():
    from orthocache_gpu_b200.synthetic import mha_inputs
    x = mha_inputs(8, 1024, 128, seed=6)
    k = T(x.keys, torch.float16).permute(1, 0, 2).contiguous()      # (S, H, hd)
    v = T(x.values, torch.float16).permute(1, 0, 2).contiguous()
    q = T(x.q, torch.float16)
    out, meta = oc.orthocache_forward(q[None], k, v, zeta_max=1.0, mode="triton_fused")
    ref, rmeta = orc.v2_attention(cast_np(x.q, torch.float16), cast_np(x.keys, torch.float16),
                                  cast_np(x.values, torch.float16), 1.0)
    assert out.shape == (1, 8, 128)
    assert meta["tile_assignment"] == "interleaved" and meta["num_tiles_fused"] == 16
    assert abs(meta["eviction_rate"] - rmeta["eviction_rate"]) < 1e-9
    assert_close(out[0], ref, torch.float16, "pipeline")


def test_v1_single_tile_and_empty_sequence():
    q = torch.randn(1, 64, device=DEV)
    k = torch.randn(64, 64, device=DEV)
    v = torch.randn(64, 64, device=DEV)
    out, meta = oc.fused_orthocache_attention(q, k, v, 1e9, return_mask=True)
    ref, _ = orc.v1_attention(as_np(q), as_np(k), as_np(v), 1e9)
    assert_close(out, ref, torch.float32, "one tile")
    out0, meta0 = oc.fused_orthocache_attention(q, k[:0], v[:0], 5.0, return_mask=True)
    assert meta0["eviction_mask"].numel() == 0 and out0.abs().max().item() == 0.0


# ------------------------------------------------------------ V3
@pytest.mark.parametrize("group", [1, 2, 4, 8, 3, 16])  # 16: two query chunks per kv head
def test_v3_groups(group):
    from orthocache_gpu_b200.synthetic import gqa_inputs
    x = gqa_inputs(2, group, 1024, 128, seed=group)
    dt = torch.bfloat16
    q, k, v = (cast_np(a, dt) for a in (x.q, x.keys, x.values))
    for tau in (1.0, 150.0):
        ref, meta = orc.v3_gqa_attention(q, k, v, tau, group)
        out, gm = oc.fused_orthocache_attention_v3_gqa(T(x.q, dt), T(x.keys, dt), T(x.values, dt), tau, group,
                                                       return_mask=True)
        near = assert_mask(gm["eviction_mask"], meta["eviction_mask"], meta["cs_bound"], tau, "v3")
        if len(near):
            ref, meta = orc.v3_gqa_attention(q, k, v, tau, group,
                                             forced=gpu_forced(gm["eviction_mask"], meta["cs_bound"], tau))
        assert gm["tiles_retained"] == meta["tiles_retained"]
        assert_close(out, ref, dt, f"v3 G={group} tau={tau}")


def test_v3_batched_extension_equals_per_sequence_calls():
    from orthocache_gpu_b200.synthetic import gqa_inputs
    x = gqa_inputs(2, 4, 512, 128, seed=21, batch=3)
    dt = torch.bfloat16
    q, k, v = T(x.q, dt), T(x.keys, dt), T(x.values, dt)
    out, meta = oc.fused_orthocache_attention_v3_gqa(q, k, v, 150.0, 4)
    assert out.shape == (3, 8, 128) and meta["num_seqs"] == 3
    for b in range(3):
        ob, _ = oc.fused_orthocache_attention_v3_gqa(q[b], k[b], v[b], 150.0, 4)
        assert (ob.float() - out[b].float()).abs().max().item() <= 1e-6


# ------------------------------------------------------------ paged
@pytest.mark.parametrize("block_size", [16, 32, 64, 128])
def test_paged_gqa_ragged_against_composed_oracle(block_size):
    from orthocache_gpu_b200.synthetic import paged_inputs
    x = paged_inputs(5, 2, 4, 128, block_size, 64, 1024, seed=block_size, extra_blocks=3)
    dt = torch.float16
    q, kc, vc, bt, sl = x.torch(dt, DEV)
    args = (cast_np(x.q, dt), cast_np(x.k_cache, dt), cast_np(x.v_cache, dt), x.block_tables)
    ref, keep, score = orc.paged_attention(*args, tau=150.0, seq_lens=x.seq_lens)
    out, meta = oc.fused_orthocache_attention_paged(q, kc, vc, bt, None, seq_lens=sl, tau=150.0,
                                                    return_mask=True)
    _check_paged_mask(meta["eviction_mask"], keep, score, 150.0, x.seq_lens, f"paged bs={block_size}")
    if orc.near_threshold(score, 150.0).any():
        ref, keep, _ = orc.paged_attention(*args, tau=150.0, seq_lens=x.seq_lens,
                                           forced=gpu_forced(meta["eviction_mask"], score, 150.0))
    assert meta["tiles_retained"] == int(keep.sum())
    assert_close(out, ref, dt, f"paged bs={block_size}")


def _check_paged_mask(mask, keep, score, thr, seq_lens, what):
    """Bit-exact on every valid tile (outside the near list); False beyond each sequence's length."""
    m = as_np(mask).astype(bool)
    valid = np.zeros(keep.shape, bool)
    for s_, n in enumerate(seq_lens):
        valid[s_, :, : int(n) // 64] = True
    assert not (m & ~valid).any(), f"{what}: mask set beyond a sequence's length"
    assert_mask(m[valid], keep[valid], score[valid], thr, what)


def test_paged_mha_zeta_equals_v2_per_sequence():
    from orthocache_gpu_b200.synthetic import paged_inputs
    x = paged_inputs(3, 4, 1, 64, 16, 512, 512, seed=2)
    dt = torch.float16
    q, kc, vc, bt, _ = x.torch(dt, DEV)
    out, _ = oc.fused_orthocache_attention_paged(q, kc, vc, bt, 1.0)
    args = (cast_np(x.q, dt), cast_np(x.k_cache, dt), cast_np(x.v_cache, dt), x.block_tables)
    _, gm = oc.fused_orthocache_attention_paged(q, kc, vc, bt, 1.0, return_mask=True)
    ref, keep, score = orc.paged_attention(*args, zeta_max=1.0)
    assert_mask(gm["eviction_mask"], keep, score, 1.0, "paged mha zeta mask")
    if orc.near_threshold(score, 1.0).any():
        ref, keep, _ = orc.paged_attention(*args, zeta_max=1.0, forced=gpu_forced(gm["eviction_mask"], score, 1.0))
    assert gm["tiles_retained"] == int(keep.sum())
    assert_close(out, ref, dt, "paged mha zeta")


def test_v3_more_units_than_one_launch():
    # 300 sequences x 8 kv heads = 2400 units: the library splits the batch
    # into launches of at most 2048 units that share one workspace
    from orthocache_gpu_b200.synthetic import gqa_inputs
    x = gqa_inputs(8, 1, 128, 64, seed=5, batch=300)
    dt = torch.float16  # two tiles a sequence: outputs near 1, where bf16 rounding alone exceeds 2e-3
    q, k, v = (cast_np(a, dt) for a in (x.q, x.keys, x.values))
    out, meta = oc.fused_orthocache_attention_v3_gqa(T(x.q, dt), T(x.keys, dt), T(x.values, dt), 100.0, 1)
    assert out.shape == (300, 8, 64)
    kept = 0
    for b in range(300):
        ref, rm = orc.v3_gqa_attention(q[b], k[b], v[b], 100.0, 1)
        kept += rm["tiles_retained"]
        assert_close(out[b], ref, dt, f"v3 batch element {b}")
    assert meta["tiles_retained"] == kept


def test_paged_batch_with_an_empty_sequence():
    from orthocache_gpu_b200.synthetic import paged_inputs
    x = paged_inputs(4, 2, 4, 128, 32, 256, 1024, seed=9)
    lens = x.seq_lens.copy()
    lens[1] = 0
    dt = torch.float16
    q, kc, vc, bt, _ = x.torch(dt, DEV)
    sl = torch.from_numpy(lens).to(DEV)
    args = (cast_np(x.q, dt), cast_np(x.k_cache, dt), cast_np(x.v_cache, dt), x.block_tables)
    ref, keep, score = orc.paged_attention(*args, tau=150.0, seq_lens=lens)
    out, meta = oc.fused_orthocache_attention_paged(q, kc, vc, bt, None, seq_lens=sl, tau=150.0, return_mask=True)
    _check_paged_mask(meta["eviction_mask"], keep, score, 150.0, lens, "paged with an empty sequence")
    if orc.near_threshold(score, 150.0).any():
        ref, keep, _ = orc.paged_attention(*args, tau=150.0, seq_lens=lens,
                                           forced=gpu_forced(meta["eviction_mask"], score, 150.0))
    assert meta["tiles_retained"] == int(keep.sum())
    assert out[1].abs().max().item() == 0.0
    assert_close(out, ref, dt, "paged with an empty sequence")


# ------------------------------------------------------------ float8 keys
# The reference's fp8 path (tests/test_fp8.py:33-127): keys quantised with
# scale = max|k| / 448, k_scale folded into q for V1 / V2 / V3; the paged path
# de-quantises the cache into q's dtype first (paged_eviction.py:355-357).
def _q_scaled(q32, scale):
    return (torch.from_numpy(np.ascontiguousarray(q32)) * scale).numpy()


@pytest.mark.parametrize("thr", [999.0, 1.0])
def test_fp8_keys_v1(thr):
    from orthocache_gpu_b200.synthetic import mha_inputs
    x = mha_inputs(1, 2048, 128, seed=31)
    k8, s = fp8_quantize(x.keys[0])
    out, meta = oc.fused_orthocache_attention(T(x.q), k8.to(DEV), T(x.values[0]), thr, return_mask=True, k_scale=s)
    kf = k8.float().numpy()
    ref, rm = orc.v1_attention(_q_scaled(x.q, s), kf, x.values[0], thr)
    assert_mask(meta["eviction_mask"], rm["eviction_mask"], rm["zeta"], thr, "v1 fp8")
    ref, rm = orc.v1_attention(_q_scaled(x.q, s), kf, x.values[0], thr,
                               forced=gpu_forced(meta["eviction_mask"], rm["zeta"], thr))
    assert meta["tiles_retained"] == rm["tiles_retained"]
    assert_close(out, ref, torch.float32, f"v1 fp8 thr={thr}")


@pytest.mark.parametrize("tau", [999.0, 150.0])
def test_fp8_keys_v3(tau):
    from orthocache_gpu_b200.synthetic import gqa_inputs
    x = gqa_inputs(2, 4, 1024, 128, seed=32)
    k8, s = fp8_quantize(x.keys)
    out, meta = oc.fused_orthocache_attention_v3_gqa(T(x.q), k8.to(DEV), T(x.values), tau, 4, return_mask=True,
                                                     k_scale=s)
    kf, qs = k8.float().numpy(), _q_scaled(x.q, s)
    ref, rm = orc.v3_gqa_attention(qs, kf, x.values, tau, 4)
    assert_mask(meta["eviction_mask"], rm["eviction_mask"], rm["cs_bound"], tau, "v3 fp8")
    ref, rm = orc.v3_gqa_attention(qs, kf, x.values, tau, 4,
                                   forced=gpu_forced(meta["eviction_mask"], rm["cs_bound"], tau))
    assert meta["tiles_retained"] == rm["tiles_retained"]
    assert_close(out, ref, torch.float32, f"v3 fp8 tau={tau}")


@pytest.mark.parametrize("qdt", [torch.float16, torch.bfloat16, torch.float32])
def test_fp8_keys_paged_dequantise_into_q_dtype(qdt):
    # reference semantics: K_eff = (k8.to(q.dtype) * k_scale) in q's dtype, q unscaled;
    # tolerance: the query dtype's (1e-5 float32, 2e-3 float16 / bfloat16)
    from orthocache_gpu_b200.synthetic import paged_inputs
    x = paged_inputs(4, 2, 4, 128, 16, 256, 1024, seed=33)
    k8, s = fp8_quantize(x.k_cache)
    keff = (k8.to(qdt) * s).float().numpy()
    q, _, vc, bt, sl = x.torch(qdt, DEV)
    out, meta = oc.fused_orthocache_attention_paged(q, k8.to(DEV), vc, bt, None, seq_lens=sl, tau=150.0,
                                                    return_mask=True, k_scale=s)
    args = (cast_np(x.q, qdt), keff, cast_np(x.v_cache, qdt), x.block_tables)
    ref, keep, score = orc.paged_attention(*args, tau=150.0, seq_lens=x.seq_lens)
    _check_paged_mask(meta["eviction_mask"], keep, score, 150.0, x.seq_lens, f"paged fp8 {qdt}")
    ref, keep, _ = orc.paged_attention(*args, tau=150.0, seq_lens=x.seq_lens,
                                       forced=gpu_forced(meta["eviction_mask"], score, 150.0))
    assert meta["tiles_retained"] == int(keep.sum())
    assert_close(out, ref, qdt, f"paged fp8 {qdt}")


# ------------------------------------------------------------ device status without a host read
def test_bad_block_table_entry_is_reported_with_stats_false():
    # an out-of-range page id: the kernel clamps the lookup to page 0 (no bad
    # access) and sets a status bit; a stats=False call cannot raise itself,
    # so the bit is visible in meta['status'] and raised by check_status()
    from orthocache_gpu_b200.synthetic import paged_inputs
    x = paged_inputs(2, 2, 1, 64, 16, 128, 256, seed=3)
    q, kc, vc, bt, _ = x.torch(torch.float16, DEV)
    oc.check_status()
    bt[0, 0] = kc.shape[0] + 5
    out, meta = oc.fused_orthocache_attention_paged(q, kc, vc, bt, 1.0, stats=False)
    assert int(meta["status"].item()) & 2
    with pytest.raises(RuntimeError, match="block-table"):
        oc.check_status()
    oc.check_status()  # the word was cleared by the read
    bt[0, 0] = -1
    with pytest.raises(RuntimeError, match="block-table"):
        oc.fused_orthocache_attention_paged(q, kc, vc, bt, 1.0)  # stats=True raises at once
