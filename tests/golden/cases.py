"""Deterministic inputs of the golden cases.

Inputs are regenerated from numpy seeds (``numpy.random.default_rng``), so the
fixtures hold only the reference's outputs plus a SHA-256 of the inputs; a
test that finds a different input hash fails instead of comparing against the
wrong vectors.  ``make_golden.py`` runs the reference on exactly these inputs.
"""

from __future__ import annotations

import hashlib

import numpy as np

from orthocache_gpu_b200.synthetic import tile_mixture, walsh

TILE = 64


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def _semantic_noise_keys(rng, n_sem, n_noise, hd):
    """Reference test pattern: semantic tiles then noise tiles (test_fused_kernel.py:195-205)."""
    w = walsh(TILE)
    blocks = []
    for _ in range(n_sem):
        coef = np.zeros((TILE, hd), np.float32)
        coef[:8] = rng.standard_normal((8, hd), dtype=np.float32) * 2.0
        blocks.append(w.T @ coef)
    for _ in range(n_noise):
        blocks.append(rng.standard_normal((TILE, hd), dtype=np.float32) * 0.1)
    return np.concatenate(blocks, 0).astype(np.float32)


def case_inputs(name: str) -> dict:
    """Inputs (float32 numpy, plus metadata) of golden case ``name``."""
    if name == "mask_semantic":
        rng = np.random.default_rng(123)
        return {"keys": _semantic_noise_keys(rng, 8, 8, 128), "thresholds": [5.0, 1.0, 0.05]}
    if name == "mask_random":
        rng = np.random.default_rng(456)
        return {"keys": rng.standard_normal((32 * TILE, 128), dtype=np.float32),
                "thresholds": [3.0, 4.5, 5.0]}
    if name == "mask_mixture_hd64":
        rng = np.random.default_rng(7)
        keys, _ = tile_mixture(rng, (), 48, 64)
        return {"keys": keys, "thresholds": [5.0, 1.0]}
    if name == "v1_config1":
        # configuration 1: q (1,128), K,V (4096,128) fp32, mixture, seed 0
        rng = np.random.default_rng(0)
        keys, _ = tile_mixture(rng, (), 64, 128)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((1, 128), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "thresholds": [5.0, 1.0, 1e9, 0.0]}
    if name == "v2_f16":
        rng = np.random.default_rng(11)
        keys, _ = tile_mixture(rng, (4,), 16, 128)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((4, 128), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "dtype": "float16",
                "thresholds": [5.0, 1.0]}
    if name == "v2_bf16_hd64":
        rng = np.random.default_rng(12)
        keys, _ = tile_mixture(rng, (3,), 10, 64)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((3, 64), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "dtype": "bfloat16",
                "thresholds": [5.0, 1.0]}
    if name == "v3_bf16":
        rng = np.random.default_rng(13)
        keys, _ = tile_mixture(rng, (2,), 12, 128)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((8, 128), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "dtype": "bfloat16", "group": 4,
                "thresholds": [1.0, 150.0, 0.0, 1e9]}
    if name == "v3_f32_g1":
        rng = np.random.default_rng(14)
        keys, _ = tile_mixture(rng, (3,), 6, 64)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((3, 64), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "dtype": "float32", "group": 1,
                "thresholds": [100.0, 0.0]}
    if name == "paged_f32":
        # reference paged test shape (test_paged_eviction.py:27-90): 2 seqs,
        # 4 heads, hd 64, block 32, 4 tiles, shuffled pool of 21 pages
        rng = np.random.default_rng(42)
        ns, nh, hd, bs, nt = 2, 4, 64, 32, 4
        seq = nt * TILE
        mb = seq // bs
        keys, _ = tile_mixture(rng, (ns, nh), nt, hd)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((ns, nh, hd), dtype=np.float32)
        total = ns * mb + 5
        perm = rng.permutation(total).astype(np.int32)
        tables = perm[: ns * mb].reshape(ns, mb).copy()
        kc = np.zeros((total, nh, bs, hd), np.float32)
        vc = np.zeros_like(kc)
        for s in range(ns):
            for b in range(mb):
                kc[tables[s, b]] = keys[s, :, b * bs:(b + 1) * bs]
                vc[tables[s, b]] = values[s, :, b * bs:(b + 1) * bs]
        return {"q": q, "k_cache": kc, "v_cache": vc, "block_tables": tables,
                "thresholds": [999.0, 1.0]}
    if name == "v2_fp8":
        # fp8 keys with k_scale folded into q (test_fp8.py:16-28 quantiser)
        rng = np.random.default_rng(15)
        keys, _ = tile_mixture(rng, (2,), 4, 64)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((2, 64), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "thresholds": [999.0, 1.0]}
    if name == "norm_cache":
        # SpectralNormCache.populate_from_keys, bands [48, 64) (the model path's) and [32, 64)
        rng = np.random.default_rng(41)
        keys, _ = tile_mixture(rng, (4,), 12, 64)
        return {"keys": keys, "thresholds": [48.0, 32.0]}
    if name == "decode_gate":
        # _pytorch_decode_gate: 4 kv heads x G 4, head_dim 64, 12 valid of 16 tiles;
        # half of the query heads high-band-zeroed; thresholds are tau values
        rng = np.random.default_rng(42)
        q = rng.standard_normal((16, 64), dtype=np.float32)
        q[1::2] = np.repeat(q[1::2].reshape(8, 8, 8).mean(-1), 8, axis=-1)  # block-constant: q_high = 0
        norms = np.abs(rng.standard_normal((4, 16), dtype=np.float32)) * 60.0
        return {"q": q, "norms": norms, "thresholds": [0.05, 0.1, 0.2]}
    if name == "hf_hook":
        # the harness's OrthoCache_GQA_Attention: prefill of 200 tokens, then
        # decode steps at 201, 255, 256 and 257 cached tokens (tile 3 completes at 256)
        rng = np.random.default_rng(43)
        keys, _ = tile_mixture(rng, (2, 2), 5, 64)                      # (B, KVH, 320, hd)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q_pre = rng.standard_normal((2, 8, 200, 64), dtype=np.float32)
        q_dec = rng.standard_normal((4, 2, 8, 1, 64), dtype=np.float32)
        return {"keys": keys, "values": values, "q_pre": q_pre, "q_dec": q_dec,
                "steps": np.array([201, 255, 256, 257]), "thresholds": [0.05]}
    if name == "compact":
        # orthocache_forward(mode='compact'): 8 blocks of 512 tokens, half of
        # them low-sequency (the first 64 rows of the 512-point Walsh basis)
        rng = np.random.default_rng(44)
        w = walsh(512)[:, :64]
        blocks = []
        for b in range(8):
            if b % 2 == 0:
                coef = rng.standard_normal((64, 4 * 64), dtype=np.float32)
                blk = w @ coef + np.float32(0.05) * rng.standard_normal((512, 4 * 64), dtype=np.float32)
            else:
                blk = rng.standard_normal((512, 4 * 64), dtype=np.float32)
            blocks.append(blk.reshape(512, 4, 64))
        keys = np.concatenate(blocks, 0).astype(np.float32)
        values = rng.standard_normal(keys.shape, dtype=np.float32)
        q = rng.standard_normal((4, 4, 64), dtype=np.float32)
        return {"q": q, "keys": keys, "values": values, "thresholds": [1.0, 5.0, 50.0]}
    raise KeyError(name)


CASES = ["mask_semantic", "mask_random", "mask_mixture_hd64", "v1_config1", "v2_f16",
         "v2_bf16_hd64", "v3_bf16", "v3_f32_g1", "paged_f32", "v2_fp8",
         "norm_cache", "decode_gate", "hf_hook", "compact"]


def fp8_quantize(keys_f32):
    """The reference tests' fp8 quantiser: scale = max|x| / 448 (test_fp8.py:16-28)."""
    import torch
    t = torch.from_numpy(keys_f32)
    max_val = t.abs().max().item()
    scale = max_val / 448.0 if max_val > 0 else 1.0
    return (t / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn), scale
