"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures in ``tests/golden`` were produced by running the reference's
CPU path on the inputs of ``tests/golden/cases.py`` (see ``make_golden.py``).
These tests prove that ``oracle/orthocache_oracle.py`` reproduces them, so the
GPU parity tests can use the oracle at sizes the reference's Python loops
cannot reach.
"""

import os

import numpy as np
import pytest
import torch

from cases import CASES, case_inputs, digest, fp8_quantize
from oracle import orthocache_oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    inp = case_inputs(name)
    arrays = [v for v in inp.values() if isinstance(v, np.ndarray)]
    assert str(z["input_sha256"]) == digest(*arrays), f"{name}: regenerated inputs drifted"
    return inp, z


def cast(a, dtype):
    return torch.from_numpy(a).to(getattr(torch, dtype)).float().numpy()


def test_walsh_matrix_properties():
    w = orc.walsh_matrix(64)
    np.testing.assert_allclose(w @ w.T, np.eye(64), atol=1e-6)
    np.testing.assert_array_equal(w, w.T)
    np.testing.assert_allclose(w[0], np.full(64, 0.125), atol=1e-7)
    assert set(np.unique(np.abs(w))) == {np.float32(0.125)}


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("mask")])
def test_mask_and_zeta_match_reference(name):
    inp, z = load(name)
    zeta = orc.tile_zeta(inp["keys"])
    for i, thr in enumerate(z["thresholds"]):
        np.testing.assert_allclose(zeta, z[f"zeta_{i}"], rtol=2e-6, atol=0)
        ref_mask = z[f"mask_{i}"]
        mask = orc.zeta_mask(zeta, thr)
        near = orc.near_threshold(z[f"zeta_{i}"], thr)
        assert np.array_equal(mask[~near], ref_mask[~near])


def test_v1_config1_matches_reference():
    inp, z = load("v1_config1")
    for i, thr in enumerate(z["thresholds"]):
        out, meta = orc.v1_attention(inp["q"], inp["keys"], inp["values"], thr)
        np.testing.assert_allclose(out, z[f"out_{i}"], atol=1e-6, rtol=0)
        near = orc.near_threshold(meta["zeta"], thr)
        assert np.array_equal(meta["eviction_mask"][~near], z[f"mask_{i}"][~near])
        assert meta["tiles_retained"] == int(z[f"retained_{i}"])


@pytest.mark.parametrize("name", ["v2_f16", "v2_bf16_hd64"])
def test_v2_matches_reference(name):
    inp, z = load(name)
    q, k, v = (cast(inp[x], inp["dtype"]) for x in ("q", "keys", "values"))
    for i, thr in enumerate(z["thresholds"]):
        out, meta = orc.v2_attention(q, k, v, thr)
        np.testing.assert_allclose(out, z[f"out32_{i}"], atol=1e-6, rtol=0)
        np.testing.assert_allclose(meta["zeta"], z[f"zeta_{i}"], rtol=2e-6)
        assert meta["tiles_retained"] == int(z[f"retained_{i}"])


@pytest.mark.parametrize("name", ["v3_bf16", "v3_f32_g1"])
def test_v3_matches_reference(name):
    inp, z = load(name)
    q, k, v = (cast(inp[x], inp["dtype"]) for x in ("q", "keys", "values"))
    for i, tau in enumerate(z["thresholds"]):
        out, meta = orc.v3_gqa_attention(q, k, v, tau, inp["group"])
        np.testing.assert_allclose(out, z[f"out32_{i}"], atol=1e-6, rtol=0)
        assert meta["tiles_retained"] == int(z[f"retained_{i}"])
        assert meta["tiles_evicted"] == int(z[f"evicted_{i}"])


def test_paged_matches_reference():
    inp, z = load("paged_f32")
    for i, thr in enumerate(z["thresholds"]):
        out, _, _ = orc.paged_attention(inp["q"], inp["k_cache"], inp["v_cache"],
                                     inp["block_tables"], zeta_max=thr)
        np.testing.assert_allclose(out, z[f"out_{i}"], atol=1e-6, rtol=0)


def test_fp8_keys_match_reference():
    inp, z = load("v2_fp8")
    k8, scale = fp8_quantize(inp["keys"])
    assert scale == float(z["k_scale"])
    assert np.array_equal(k8.view(torch.uint8).numpy(), z["keys_fp8_bits"])
    kf = k8.float().numpy()
    q = (torch.from_numpy(inp["q"]) * scale).numpy()     # k_scale folded into q
    for i, thr in enumerate(z["thresholds"]):
        out, _ = orc.v2_attention(q, kf, inp["values"], thr)
        np.testing.assert_allclose(out, z[f"out_{i}"], atol=1e-6, rtol=0)


def test_lse_merge_equals_unsplit():
    rng = np.random.default_rng(3)
    hd, s = 16, 5
    logits = rng.standard_normal((s, 7)) * 3
    vals = rng.standard_normal((s, 7, hd))
    m = logits.max(1)
    p = np.exp(logits - m[:, None])
    l = p.sum(1)
    acc = np.einsum("st,std->sd", p, vals)
    m[2], l[2], acc[2] = -1e9, 0.0, 0.0               # an empty split
    full = np.concatenate([np.exp(logits[i] - logits.max()) for i in range(s) if i != 2])
    v = np.concatenate([vals[i] for i in range(s) if i != 2])
    np.testing.assert_allclose(orc.lse_merge(m, l, acc), full @ v / full.sum(), atol=1e-12)
    # all splits empty -> zeros
    np.testing.assert_array_equal(orc.lse_merge(np.full(3, -1e9), np.zeros(3), np.zeros((3, hd))),
                                  np.zeros(hd))


def test_norm_cache_matches_reference():
    inp, z = load("norm_cache")
    for i, hs in enumerate(z["thresholds"]):
        norms = orc.tile_high_norms(inp["keys"], int(hs), 64)
        ref = z[f"norms_{i}"]
        np.testing.assert_allclose(norms, ref[:, :12], rtol=2e-6, atol=0)
        assert not ref[:, 12:].any() and (z[f"valid_{i}"] == 12).all()


# |q_high| = sqrt(|q|^2 - |q_low|^2) cancels for queries without high band:
# float32 summation order alone leaves sqrt(~1e-7 * |q|^2) ~ 3e-3 absolute there
QH_ATOL = 4e-3


def test_decode_gate_matches_reference():
    inp, z = load("decode_gate")
    np.testing.assert_allclose(orc.q_high_norm(inp["q"]), z["q_high"], rtol=1e-5, atol=QH_ATOL)
    for i, tau in enumerate(z["thresholds"]):
        for tight in (True, False):
            evict, s, bound = orc.decode_gate(inp["q"], inp["norms"], tau, 12, 4, tight=tight)
            np.testing.assert_allclose(s, z[f"qn_{i}_{int(tight)}"], rtol=1e-5, atol=QH_ATOL)
            ref = z[f"evict_{i}_{int(tight)}"]
            near = orc.near_threshold(bound, tau * 64 * 64)
            assert np.array_equal(evict[~near], ref[~near]), (tau, tight)
            assert not ref[:, 12:].any()
