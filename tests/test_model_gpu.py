"""Llama-shaped decode with the fused kernel in every layer (small shape).

With tau = 0 the Cauchy-Schwarz gate retains every tile (bounds are > 0), so
the fused decode (kernel over whole tiles + dense ragged tail + LSE merge)
must reproduce dense decode attention; with the median-calibrated tau about
half the tiles are evicted and decoding stays finite.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = dict(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=64, mlp=512, vocab=1000)


def _model(max_len):
    from orthocache_gpu_b200.model import GatedLlama, LlamaShape
    return GatedLlama(LlamaShape(**SHAPE), max_len=max_len, seed=1)


def test_tau_zero_matches_dense_decode():
    m = _model(512)
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    prompt = torch.randint(0, SHAPE["vocab"], (300,), generator=g, device="cuda")
    logits = {}
    for mode in (None, 0.0):
        m.length = 0
        m.tau = [None] * SHAPE["layers"]
        first = m.prefill(prompt)
        tok = first.argmax(-1)
        steps = []
        for _ in range(6):   # crosses no tile boundary and one ragged tail each step
            lg = m.step(tok, mode)
            steps.append(lg.float())
        logits[mode] = torch.cat(steps)
    err = (logits[None] - logits[0.0]).abs().max().item()
    scale = logits[None].abs().max().item()
    assert err <= 2e-2 * scale + 1e-3, (err, scale)


def test_median_tau_generates():
    m = _model(1024)
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    prompt = torch.randint(0, SHAPE["vocab"], (640,), generator=g, device="cuda")
    res = m.generate(prompt, 8, tau_mode="median")
    assert len(res["tokens"]) == 9 and res["final_length"] == 648
    assert all(t is not None and t > 0 for t in res["tau"])
    assert res["ms_per_token"] > 0


def test_device_length_step_matches_eager_step_and_graph_generation_runs():
    m = _model(1024)
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    prompt = torch.randint(0, SHAPE["vocab"], (700,), generator=g, device="cuda")
    m.length = 0
    m.tau = [None] * SHAPE["layers"]
    tok = m.prefill(prompt).argmax(-1)
    m.step(tok, "median")                        # calibrates tau, length 701
    kc = [k.clone() for k in m.k_cache]
    vc = [v.clone() for v in m.v_cache]
    n0 = m.length
    ref = m.step(tok, "median").float()           # eager step at length 701 -> 702
    for i in range(SHAPE["layers"]):
        m.k_cache[i].copy_(kc[i])
        m.v_cache[i].copy_(vc[i])
    npos = torch.full((1,), n0, dtype=torch.long, device="cuda")
    t = tok.reshape(1).clone()
    got = m._step_dev(t, npos).float()
    assert int(npos) == n0 + 1
    err = (got - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err
    res = m.generate_graph(prompt, 20, tau_mode="median")
    assert len(res["tokens"]) == 21 and res["final_length"] == 700 + 20 and res["ms_per_token"] > 0


def test_flash_dense_arm_matches_sdpa_dense():
    m = _model(512)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    prompt = torch.randint(0, SHAPE["vocab"], (200,), generator=g, device="cuda")
    outs = {}
    for mode in (None, "flash"):
        m.length = 0
        tok = m.prefill(prompt).argmax(-1)
        outs[mode] = m.step(tok, mode).float()
    assert (outs[None] - outs["flash"]).abs().max().item() <= 2e-2 * outs[None].abs().max().item() + 1e-3
