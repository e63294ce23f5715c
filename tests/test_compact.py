"""orthocache_forward(mode='compact'): the 512-token block path.

Pinned to golden vectors made by the reference's own pipeline
(tests/golden case ``compact``, pipeline.py:459-555).  CPU: the host-side
spectral analysis (ζ, logit bounds, auto tau, block mask, perfect-eviction
counts).  GPU: the whole mode, whose attention runs in the library's kernel
over the retained blocks only; outputs are bfloat16 like the reference's, so
they are compared within one bfloat16 step (2^-8 relative) plus 1e-3.
"""

import numpy as np
import pytest
import torch

import orthocache_gpu_b200 as oc
from cases import case_inputs
from helpers import golden
from orthocache_gpu_b200 import compact as cp


def _inputs():
    inp, z = case_inputs("compact"), golden("compact")
    return inp, z, torch.from_numpy(inp["q"]), torch.from_numpy(inp["keys"]), torch.from_numpy(inp["values"])


def test_spectral_analysis_matches_reference():
    inp, z, q, k, _ = _inputs()
    np.testing.assert_allclose(cp.compute_spectral_decay_ratio(k).numpy(), z["zeta"], rtol=1e-4)
    np.testing.assert_allclose(cp.compute_query_aware_bounds(q, k).numpy(), z["bounds"], rtol=1e-4, atol=1e-4)
    assert abs(cp.auto_tau(q, k) - float(z["tau_0"])) < 1e-3 * abs(float(z["tau_0"]))
    for i, (zm, tau) in enumerate(z["runs"]):
        t = float(z["tau_0"]) if np.isnan(tau) else float(tau)
        m = cp.compute_multiband_mask(q, k, t, float(zm))
        assert int(torch.any(m, -1).sum()) == int(z[f"blocks_retained_{i}"])


def test_fwht_512_is_the_normalised_walsh_transform():
    from oracle import orthocache_oracle as orc
    x = torch.randn(512, 3, generator=torch.Generator().manual_seed(0))
    np.testing.assert_allclose(cp.fwht_512(x).numpy(), orc.walsh_matrix(512) @ x.numpy(), atol=1e-5)


@pytest.mark.gpu
def test_compact_mode_matches_reference_golden():
    inp, z, q, k, v = _inputs()
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    for i, (zm, tau) in enumerate(z["runs"]):
        out, meta = oc.orthocache_forward(q, k, v, mode="compact", zeta_max=float(zm),
                                          tau=None if np.isnan(tau) else float(tau))
        assert meta["actual_mode"] == "compact" and meta["blocks_retained"] == int(z[f"blocks_retained_{i}"])
        assert meta["compact_num_active"] == meta["blocks_retained"]
        for key in ("perfect_eviction_blocks", "statistical_eviction_blocks"):
            assert meta[key] == int(z[f"{key}_{i}"]), key
        for key in ("tau", "zeta_mean", "zeta_min", "zeta_max_observed"):
            assert abs(meta[key] - float(z[f"{key}_{i}"])) <= 1e-4 * max(1.0, abs(float(z[f"{key}_{i}"]))), key
        ref = z[f"out_{i}"]
        got = out.float().cpu().numpy()
        assert out.shape == (4, 4, 64)
        assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-3), f"run {i}"


@pytest.mark.gpu
def test_block_attention_long_query_batch_and_bfloat16_inputs():
    # more query positions than one launch holds (chunked), bf16 K / V
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(300, 8, 64, device="cuda", generator=g)
    k = torch.randn(2048, 8, 64, device="cuda", generator=g).bfloat16()
    v = torch.randn(2048, 8, 64, device="cuda", generator=g).bfloat16()
    mask = torch.tensor([True, False, True, True], device="cuda")
    out, st = cp.block_attention(q, k, v, mask)
    keep = mask.repeat_interleave(512)
    ref = torch.softmax(torch.einsum("qhd,khd->hqk", q, k[keep].float()) / 8.0, -1)
    ref = torch.einsum("hqk,khd->qhd", ref, v[keep].float())
    assert st["num_active"] == 3
    assert (out.float() - ref).abs().max().item() <= 1e-2
