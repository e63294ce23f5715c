"""Generate the golden fixtures by running the reference's own CPU path.

Run in a container where the reference source tree is available::

    python tests/golden/make_golden.py /path/to/orthocache-gpu

It imports ``orthocache_gpu`` from ``<ref>/src`` and calls the reference's
CPU implementations (the ``_pytorch_*`` functions its public wrappers use
without CUDA) on the inputs of ``cases.py``.  Outputs are stored in
``tests/golden/<case>.npz`` together with the SHA-256 of the inputs.  The
GPU box never runs this script; the tests only read the ``.npz`` files.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)


def main(ref_root: str, only=None) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from orthocache_gpu.triton_kernels import fwht_fused_prototype as fw
    from orthocache_gpu.triton_kernels import fused_eviction as fe
    from orthocache_gpu.triton_kernels import gqa_eviction as ge
    from orthocache_gpu.triton_kernels import paged_eviction as pe

    from cases import CASES, case_inputs, digest, fp8_quantize

    torch.set_flush_denormal(True)   # the reference's conftest does the same
    torch.set_num_threads(1)
    T = torch.from_numpy

    for name in (only or CASES):
        inp = case_inputs(name)
        out = {}
        arrays = [v for v in inp.values() if isinstance(v, np.ndarray)]
        out["input_sha256"] = np.array(digest(*arrays))
        out["torch_version"] = np.array(torch.__version__)
        ths = inp["thresholds"]
        out["thresholds"] = np.array(ths, np.float64)
        if name.startswith("mask"):
            for i, z in enumerate(ths):
                m, zeta = fw._pytorch_fwht_eviction(T(inp["keys"]), z, return_zeta=True)
                out[f"mask_{i}"] = m.numpy()
                out[f"zeta_{i}"] = zeta.numpy()
        elif name == "v1_config1":
            for i, z in enumerate(ths):
                o, meta = fe.fused_orthocache_attention(
                    T(inp["q"]), T(inp["keys"]), T(inp["values"]), z, return_mask=True)
                out[f"out_{i}"] = o.numpy()
                out[f"mask_{i}"] = meta["eviction_mask"].numpy()
                out[f"retained_{i}"] = np.array(meta["tiles_retained"])
        elif name in ("v2_f16", "v2_bf16_hd64"):
            dt = getattr(torch, inp["dtype"])
            q, k, v = (T(inp[x]).to(dt) for x in ("q", "keys", "values"))
            for i, z in enumerate(ths):
                # internal CPU path keeps the fp32 output (public wrapper casts to dtype)
                o32, meta = fe._pytorch_fused_orthocache_multihead(q, k, v, z)
                o, _ = fe.fused_orthocache_attention_v2(q, k, v, z)
                out[f"out32_{i}"] = o32.numpy()
                out[f"out_{i}"] = o.float().numpy()
                out[f"retained_{i}"] = np.array(meta["tiles_retained"])
                masks = [fw._pytorch_fwht_eviction(k[h], z, return_zeta=True) for h in range(k.shape[0])]
                out[f"zeta_{i}"] = np.stack([m[1].numpy() for m in masks])
        elif name.startswith("v3"):
            dt = getattr(torch, inp["dtype"])
            q, k, v = (T(inp[x]).to(dt) for x in ("q", "keys", "values"))
            g = inp["group"]
            for i, tau in enumerate(ths):
                o32, meta = ge._pytorch_gqa_cauchy_schwarz_attention(q, k, v, tau, g)
                o, _ = ge.fused_orthocache_attention_v3_gqa(q, k, v, tau, g)
                out[f"out32_{i}"] = o32.numpy()
                out[f"out_{i}"] = o.float().numpy()
                out[f"retained_{i}"] = np.array(meta["tiles_retained"])
                out[f"evicted_{i}"] = np.array(meta["tiles_evicted"])
        elif name == "paged_f32":
            q, kc, vc = T(inp["q"]), T(inp["k_cache"]), T(inp["v_cache"])
            bt = T(inp["block_tables"])
            for i, z in enumerate(ths):
                o, _ = pe.fused_orthocache_attention_paged(q, kc, vc, bt, z)
                out[f"out_{i}"] = o.numpy()
        elif name == "v2_fp8":
            k8, scale = fp8_quantize(inp["keys"])
            q, v = T(inp["q"]), T(inp["values"])
            out["k_scale"] = np.array(scale)
            out["keys_fp8_bits"] = k8.view(torch.uint8).numpy()
            for i, z in enumerate(ths):
                o, _ = fe.fused_orthocache_attention_v2(q, k8, v, z, k_scale=scale)
                out[f"out_{i}"] = o.numpy()
        elif name == "norm_cache":
            from orthocache_gpu import norm_cache as ncm
            k = T(inp["keys"])
            w = fw.generate_walsh_matrix(64)
            for i, hs in enumerate(ths):
                c = ncm.SpectralNormCache(4, 16, torch.device("cpu"))
                c.populate_from_keys(k, w, high_start=int(hs), high_end=64)
                out[f"norms_{i}"] = c.cache.numpy()
                out[f"valid_{i}"] = c.valid_tiles.numpy()
        elif name == "decode_gate":
            from orthocache_gpu.triton_kernels import decode_gate as dg
            q, nrm = T(inp["q"]), T(inp["norms"])
            out["q_high"] = dg.compute_q_high_norm_exact(q).numpy()
            for i, tau in enumerate(ths):
                for tight in (True, False):
                    m, qn = dg._pytorch_decode_gate(q, nrm, tau, 12, 4, 64, tight=tight)
                    out[f"evict_{i}_{int(tight)}"] = m.numpy()
                    out[f"qn_{i}_{int(tight)}"] = qn.numpy()
        elif name == "hf_hook":
            sys.path.insert(0, os.path.join(ref_root, "eval"))
            import perplexity_eval as pev
            from orthocache_gpu.norm_cache import SpectralNormCache
            oca = pev.OrthoCache_GQA_Attention(tau=ths[0])
            oca.norm_cache = SpectralNormCache(2, 8, torch.device("cpu"))
            k, v = T(inp["keys"]), T(inp["values"])
            out["prefill"] = oca.orthocache_attention(T(inp["q_pre"]), k[:, :, :200], v[:, :, :200], 4).numpy()
            out["prefill_evicted"] = np.array(oca.stats["evicted_tiles"])
            out["norms"] = oca.norm_cache.cache.numpy()
            for i, n in enumerate(inp["steps"]):
                before = oca.stats["decode_tiles_skipped"]
                out[f"decode_{i}"] = oca.orthocache_attention(T(inp["q_dec"][i]), k[:, :, :n], v[:, :, :n], 4).numpy()
                out[f"decode_skipped_{i}"] = np.array(oca.stats["decode_tiles_skipped"] - before)
        elif name == "compact":
            # the reference's torch.compile wrappers need a host compiler: run them
            # eagerly (TORCHDYNAMO_DISABLE=1 in the environment) -- same arithmetic
            from orthocache_gpu import pipeline as ppl
            from orthocache_gpu import spectral_energy as se
            q, k, v = T(inp["q"]), T(inp["keys"]), T(inp["values"])
            out["zeta"] = se.compute_spectral_decay_ratio(k).numpy()
            out["bounds"] = se.compute_query_aware_bounds(q, k).numpy()
            runs = [(1.0, None), (5.0, None), (50.0, 30.0), (50.0, 1e9)]
            out["runs"] = np.array([[z, np.nan if t is None else t] for z, t in runs])
            for i, (zm, tau) in enumerate(runs):
                o, meta = ppl.orthocache_forward(q, k, v, mode="compact", zeta_max=zm, tau=tau)
                out[f"out_{i}"] = o.float().numpy()
                for key in ("tau", "zeta_mean", "zeta_std", "zeta_min", "zeta_max_observed", "blocks_retained",
                            "perfect_eviction_blocks", "statistical_eviction_blocks", "perfect_eviction_rate",
                            "eviction_rate"):
                    out[f"{key}_{i}"] = np.array(meta[key])
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print("wrote", name)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference project root> [case ...]")
    main(sys.argv[1], sys.argv[2:] or None)
