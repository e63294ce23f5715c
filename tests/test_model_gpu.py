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


def _gemv_ref(x, y, norm_w, W, eps=1e-5):
    """PyTorch reference of oc_gemv's prologue (residual add + RMSNorm) and product, fp32 accumulate.

    W is (out_features, in_features)."""
    v = x if y is None else (x.float() + y.float()).to(x.dtype)
    h = v if norm_w is None else \
        (v.float() * torch.rsqrt(v.float().pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * norm_w
    return v, (h.float() @ W.float().t())


@pytest.mark.parametrize("K,N,norm,epi", [(2048, 3072, True, 0), (2048, 2048, False, 0), (5632, 2048, False, 0),
                                          (2048, 11264, True, 1), (2048, 32000, True, 0), (96, 264, False, 0),
                                          (4104, 6, True, 1)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemv_matches_torch(K, N, norm, epi, dt):
    from orthocache_gpu_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda")
    g.manual_seed(K + N)
    x = torch.randn(1, K, device="cuda", generator=g).to(dt)
    y = torch.randn(1, K, device="cuda", generator=g).to(dt) if norm else None
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(dt) if norm else None
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).to(dt)
    out = torch.empty(1, N // 2 if epi else N, device="cuda", dtype=dt)
    xo = torch.empty_like(x) if norm else None
    st = _lib.stream_ptr(x.device)
    _lib.check(lib.oc_gemv(x.data_ptr(), _lib.ptr(y), _lib.ptr(nw), 1e-5, _lib.ptr(xo), W.data_ptr(), K, K, N,
                           out.data_ptr(), epi, _lib.dtype_code(x), st), "oc_gemv")
    torch.cuda.synchronize()
    v, ref = _gemv_ref(x, y, nw, W)
    if epi:   # rows 2j / 2j + 1 are a_j / b_j
        ab = ref.to(dt).view(1, -1, 2)
        ref = (torch.nn.functional.silu(ab[..., 0]) * ab[..., 1]).float()
    if xo is not None:
        assert torch.equal(xo, v)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


def test_gemv_qkv_rope_matches_rope_append():
    from orthocache_gpu_b200 import _lib
    from orthocache_gpu_b200.model import _rope_tables
    lib = _lib.load()
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    dt, H, KVH, hd, K, T = torch.bfloat16, 8, 2, 64, 256, 128
    N = (H + 2 * KVH) * hd
    x = torch.randn(1, K, device="cuda", generator=g).to(dt)
    nw = torch.ones(K, device="cuda", dtype=dt)
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).to(dt)
    cos, sin = _rope_tables(T, hd, 10000.0, torch.device("cuda"))
    pos = torch.tensor([37], device="cuda", dtype=torch.long)
    st = _lib.stream_ptr(x.device)
    q = torch.empty(H, hd, device="cuda", dtype=dt)
    kc = torch.zeros(T, KVH, hd, device="cuda", dtype=dt)
    vc = torch.zeros_like(kc)
    xo = torch.empty_like(x)
    _lib.check(lib.oc_gemv_qkv_rope(x.data_ptr(), 0, nw.data_ptr(), 1e-5, xo.data_ptr(), W.data_ptr(), K, K,
                                    H, KVH, hd, cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), q.data_ptr(),
                                    kc.data_ptr(), vc.data_ptr(), KVH * hd, _lib.dtype_code(x), st),
               "oc_gemv_qkv_rope")
    # reference: the same projection by torch, then the rotary / append kernel
    _, ref = _gemv_ref(x, None, nw, W)
    qkv = ref.to(dt)
    q2 = torch.empty_like(q)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    _lib.check(lib.oc_rope_cache_append(qkv.data_ptr(), H, KVH, hd, cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
                                        q2.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), KVH * hd, _lib.dtype_code(x),
                                        st), "oc_rope_cache_append")
    torch.cuda.synchronize()
    for a, b in ((q, q2), (kc, kc2), (vc, vc2)):   # fp32 sums in another order: within a few 16-bit steps
        assert (a.float() - b.float()).abs().max().item() <= 2e-2 * b.float().abs().max().item() + 1e-3
    assert kc[37].abs().sum() > 0 and vc[37].abs().sum() > 0 and kc[36].abs().sum() == 0
