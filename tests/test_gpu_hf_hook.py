"""The transformers attention hook (OrthoCache_GQA_Attention, patch_model_attention).

* against golden vectors made by the reference harness's own class
  (eval/perplexity_eval.py:320-690, tests/golden/make_golden.py case
  ``hf_hook``): a 200-token prefill, then decode steps at 201, 255, 256 and
  257 cached tokens; outputs within 1e-5 (float32), evicted counts equal;
* inside a random-init transformers Llama: with tau < 0 nothing is evicted
  and the patched model's logits equal the unpatched model's; with a positive
  tau decoding runs through the cached-norm kernel and evicts tiles.
"""

import numpy as np
import pytest
import torch

from cases import case_inputs
from helpers import as_np, golden
from orthocache_gpu_b200.hf_hook import OrthoCache_GQA_Attention, patch_model_attention
from orthocache_gpu_b200.norm_cache import SpectralNormCache

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_hook_matches_reference_harness_golden():
    inp, z = case_inputs("hf_hook"), golden("hf_hook")
    oca = OrthoCache_GQA_Attention(tau=float(z["thresholds"][0]))
    oca.norm_cache = SpectralNormCache(2, 8, DEV)
    k, v = T(inp["keys"]), T(inp["values"])
    out = oca.orthocache_attention(T(inp["q_pre"]), k[:, :, :200], v[:, :, :200], 4)
    np.testing.assert_allclose(as_np(out), z["prefill"], atol=1e-5, rtol=0)
    assert oca.stats["evicted_tiles"] == int(z["prefill_evicted"])
    np.testing.assert_allclose(as_np(oca.norm_cache.cache), z["norms"], rtol=1e-5)
    for i, n in enumerate(inp["steps"]):
        before = oca.stats["decode_tiles_skipped"]
        out = oca.orthocache_attention(T(inp["q_dec"][i]), k[:, :, :n], v[:, :, :n], 4)
        assert out.shape == (2, 8, 1, 64)
        np.testing.assert_allclose(as_np(out), z[f"decode_{i}"], atol=1e-5, rtol=0, err_msg=f"decode at {n}")
        assert oca.stats["decode_tiles_skipped"] - before == int(z[f"decode_skipped_{i}"])


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=1024,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(DEV).float().eval()


def _greedy(model, ids, steps):
    with torch.no_grad():
        out = model(ids, use_cache=True)
        past, logits = out.past_key_values, [out.logits[:, -1]]
        tok = out.logits[:, -1:].argmax(-1)
        for _ in range(steps):
            out = model(tok, past_key_values=past, use_cache=True)
            past = out.past_key_values
            logits.append(out.logits[:, -1])
            tok = out.logits[:, -1:].argmax(-1)
    return torch.stack(logits, 1)


def test_patched_transformers_llama_decodes_through_the_kernel():
    pytest.importorskip("transformers")
    ids = torch.randint(0, 512, (1, 300), generator=torch.Generator().manual_seed(1)).to(DEV)
    ref = _greedy(_tiny_llama(), ids, 8)
    model = _tiny_llama()
    oca = OrthoCache_GQA_Attention(tau=-1.0)          # nothing evicted: must equal dense attention
    oca.norm_cache = SpectralNormCache(2, 16, DEV)
    patch_model_attention(model, oca)
    got = _greedy(model, ids, 8)
    assert oca.stats["decode_steps"] == 8 * 3 and oca.stats["decode_tiles_skipped"] == 0
    assert (got - ref).abs().max().item() < 2e-3
    model2 = _tiny_llama()
    oca2 = OrthoCache_GQA_Attention(tau=1e-3, refresh_norms=True)
    oca2.norm_cache = SpectralNormCache(2, 16, DEV)
    patch_model_attention(model2, oca2)
    out = _greedy(model2, ids, 8)
    assert torch.isfinite(out).all() and oca2.stats["decode_tiles_total"] > 0
