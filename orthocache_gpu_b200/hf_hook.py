"""OrthoCache attention inside a Hugging Face (transformers) Llama-family model.

Drop-in for ``OrthoCache_GQA_Attention`` and ``patch_model_attention`` of
the reference's evaluation harness (j-arndt/orthocache-gpu,
eval/perplexity_eval.py:320-745).  The patched attention layers route their
scaled-dot-product attention call here:

* prefill (more than one query position): every 64-token key tile is scored
  once on the GPU (``tile_high_norms``, |K_high|_F over Walsh rows [48, 64),
  the harness's band and its unnormalised Walsh scale), the norm cache is filled, and a tile is evicted for
  the whole query group when median_pos(|q_g|) (max over the group) times
  |K_high|_F / (64 * head_dim) <= tau; attention is dense and causal with
  the evicted tiles masked (perplexity_eval.py:404-551);
* decode (one query position, norm cache populated): the O(1) cached-norm
  gate with the median over the group of the exact |q_high| and the fused
  kernel over the retained tiles only -- evicted tiles are not read at all;
  the tokens after the last whole tile are attended densely and merged by
  log-sum-exp (perplexity_eval.py:554-674, which masks logits of a dense
  product instead).

Tiles completed during decoding: the reference never adds their norms (the
cache keeps 0 there, so they are evicted whenever tau >= 0).  That is the
default here too; ``refresh_norms=True`` scores each newly completed tile
before the gate reads it.

Norm caches: the harness shares one ``norm_cache`` among all patched layers,
so every layer's decode gate reads the norms of the last layer's keys.
``per_layer_norms=True`` (the default here) gives each patched layer its own
cache of the same capacity (created on first use); ``False`` keeps the
harness's single shared cache.

The residual governor of the harness is not part of this path (``governor`` is accepted and used only
for ``get_tau_effective`` / ``report_layer`` if given).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from .decode_gate import cached_partials
from .distributed import merge_states
from .norm_cache import SpectralNormCache, tile_high_norms

TILE = 64
HIGH_BAND = (48, 64)  # top quarter of the 64 Walsh rows (perplexity_eval.py:436-437)
# the harness's Walsh matrix is the unnormalised +-1 Hadamard matrix
# (perplexity_eval.py:54-62), so its norms are 8x those of the 1/8-scaled
# transform that tile_high_norms applies (an exact power-of-two factor)
HARNESS_NORM_SCALE = 8.0
LOG2E = 1.4426950408889634


class OrthoCache_GQA_Attention:
    """Spectral-gated attention for patched Llama attention layers (perplexity_eval.py:320-370)."""

    def __init__(self, tau: float = 1.0, verbose: bool = False, governor=None, refresh_norms: bool = False,
                 collect_stats: bool = True, per_layer_norms: bool = True):
        self.tau = tau
        self.verbose = verbose
        self.governor = governor
        self.refresh_norms = refresh_norms
        self.collect_stats = collect_stats
        self.per_layer_norms = per_layer_norms
        self.norm_cache: Optional[SpectralNormCache] = None
        self._layer_caches: dict = {}
        self.reset_stats()

    def _cache_for(self, layer):
        nc = self.norm_cache
        if nc is None or layer is None or not self.per_layer_norms:
            return nc
        c = self._layer_caches.get(layer)
        if c is None:
            c = self._layer_caches[layer] = SpectralNormCache(nc.num_kv_heads, nc.max_tiles, nc.cache.device)
        return c

    def reset_stats(self):
        self.stats = {"total_tiles": 0, "evicted_tiles": 0, "layers_processed": 0, "cs_bounds": [],
                      "hallucination_scores": [], "q_search_intensity": [], "k_info_density": [],
                      "decode_steps": 0, "decode_tiles_skipped": 0, "decode_tiles_total": 0}

    @property
    def eviction_rate(self) -> float:
        if self.stats["total_tiles"] == 0:
            return 0.0
        return self.stats["evicted_tiles"] / self.stats["total_tiles"]

    def _tau(self) -> float:
        return self.governor.get_tau_effective(self.tau) if self.governor is not None else self.tau

    # ---------------------------------------------------------------- dispatch
    def orthocache_attention(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                             num_query_groups: int, layer: Optional[int] = None) -> torch.Tensor:
        """query (B, Hq, Sq, hd); key / value (B, KVH, S, hd) -> (B, Hq, Sq, hd) in query's dtype."""
        nc = self._cache_for(layer)
        G = num_query_groups
        if G > 1 and key.shape[1] == query.shape[1]:  # the caller already repeated the kv heads
            key, value = key[:, ::G], value[:, ::G]
        seq_len_q, seq_len_kv = query.shape[2], key.shape[2]
        if seq_len_kv < TILE:
            return self._dense_attention(query, key, value, G)
        if seq_len_q == 1 and nc is not None and nc.is_populated:
            return self._decode_attention(query, key, value, G, nc)
        return self._prefill_attention(query, key, value, G, nc)

    # ---------------------------------------------------------------- prefill
    def _prefill_attention(self, query, key, value, G, nc):
        B, Hq, Sq, hd = query.shape
        kvh, S = key.shape[1], key.shape[2]
        T = S // TILE
        nf = float(TILE * hd)
        tau = self._tau()
        outs = []
        for b in range(B):
            q_b, k_b, v_b = query[b].float(), key[b].float(), value[b].float()
            knorm = tile_high_norms(k_b[:, : T * TILE], *HIGH_BAND) * HARNESS_NORM_SCALE  # (KVH, T) float32
            if nc is not None:
                t_ = min(T, nc.max_tiles)
                nc.cache[:kvh, :t_] = knorm[:, :t_]
                nc.valid_tiles[:kvh].clamp_(min=t_)
                nc._populated = True
            qmed = torch.linalg.vector_norm(q_b, dim=-1).median(dim=1).values           # (Hq,) lower median
            qmax = qmed.view(kvh, G).amax(1)
            # the harness compares Python floats: (float32 * float32) / nf <= tau in double precision
            evict = (qmax.double()[:, None] * knorm.double()) / nf <= tau                # (KVH, T)
            k_e = k_b.repeat_interleave(G, 0)
            v_e = v_b.repeat_interleave(G, 0)
            logits = torch.matmul(q_b, k_e.transpose(-2, -1)) * (1.0 / math.sqrt(hd))
            causal = torch.ones(Sq, S, device=query.device, dtype=torch.bool).triu(1 + S - Sq)
            tok = torch.zeros(kvh, S, dtype=torch.bool, device=query.device)
            tok[:, : T * TILE] = evict.repeat_interleave(TILE, 1)
            logits.masked_fill_(causal[None] | tok.repeat_interleave(G, 0)[:, None, :], float("-inf"))
            w = torch.nan_to_num(F.softmax(logits, dim=-1), nan=0.0)
            outs.append(torch.matmul(w, v_e).to(query.dtype))
            if self.collect_stats:
                n_ev = int(evict.sum())
                self.stats["total_tiles"] += T * kvh
                self.stats["evicted_tiles"] += n_ev
                if self.governor is not None and T > 0:
                    self.governor.report_layer(n_ev / (T * kvh))
                if T > 0:
                    mq, mk = float(qmax.max()), float(knorm.max())
                    self.stats["hallucination_scores"].append(mq / (mk + 1e-10))
                    self.stats["q_search_intensity"].append(mq)
                    self.stats["k_info_density"].append(mk)
        self.stats["layers_processed"] += 1
        return torch.stack(outs, 0)

    # ---------------------------------------------------------------- decode
    def _decode_attention(self, query, key, value, G, nc):
        B, Hq, _, hd = query.shape
        kvh, S = key.shape[1], key.shape[2]
        T = S // TILE
        tau = self._tau()
        if T > nc.max_tiles:
            raise ValueError(f"{T} tiles exceed the norm cache's max_tiles ({nc.max_tiles})")
        if self.refresh_norms:
            valid = int(nc.valid_tiles[:kvh].min())
            if valid < T:
                tile_high_norms(key[0, :, valid * TILE: T * TILE], *HIGH_BAND, out=nc.cache[:kvh, valid:])
                nc.cache[:kvh, valid:T] *= HARNESS_NORM_SCALE
                nc.valid_tiles[:kvh].clamp_(min=T)
        norms = nc.cache[:kvh].unsqueeze(0).expand(B, kvh, nc.max_tiles)
        q = query[:, :, 0]                                                              # (B, Hq, hd)
        (m, l, acc), meta = cached_partials(q, key[:, :, : T * TILE], value[:, :, : T * TILE], norms, tau, G,
                                            tight=True, q_stat="median", stats=self.collect_stats)
        ms, ls, accs = [m], [l], [acc]
        if S > T * TILE:  # the ragged tail is always attended
            kt = key[:, :, T * TILE:].repeat_interleave(G, 1).float()                   # (B, Hq, r, hd)
            vt = value[:, :, T * TILE:].repeat_interleave(G, 1).float()
            sc = (kt @ q.float()[..., None])[..., 0] * (LOG2E / math.sqrt(hd))          # (B, Hq, r), log2 units
            mt = sc.amax(-1)
            pt = torch.exp2(sc - mt[..., None])
            ms.append(mt)
            ls.append(pt.sum(-1))
            accs.append((pt[..., None, :] @ vt)[..., 0, :])
        out = merge_states(torch.stack(ms, -1).reshape(B * Hq, -1).contiguous(),
                           torch.stack(ls, -1).reshape(B * Hq, -1).contiguous(),
                           torch.stack(accs, -2).reshape(B * Hq, -1, hd).contiguous(), query.dtype)
        if self.collect_stats:
            skipped = meta["tiles_evicted"]
            self.stats["decode_steps"] += B
            self.stats["decode_tiles_skipped"] += skipped
            self.stats["decode_tiles_total"] += T * kvh * B
            if self.governor is not None and T > 0:
                self.governor.report_layer(skipped / (T * kvh * B))
        self.stats["layers_processed"] += 1
        return out.view(B, Hq, 1, hd)

    def _dense_attention(self, query, key, value, G):
        """Dense causal attention (perplexity_eval.py:676-690)."""
        k = key.repeat_interleave(G, dim=1)
        v = value.repeat_interleave(G, dim=1)
        logits = torch.matmul(query, k.transpose(-2, -1)) * (1.0 / math.sqrt(query.shape[-1]))
        sq, skv = query.shape[2], key.shape[2]
        mask = torch.ones(sq, skv, device=query.device, dtype=torch.bool).triu(1 + skv - sq)
        logits.masked_fill_(mask, float("-inf"))
        return torch.matmul(F.softmax(logits, dim=-1), v)


def patch_model_attention(model, orthocache: OrthoCache_GQA_Attention, min_layer: int = 0):
    """Route the SDPA call of the attention layers >= min_layer through ``orthocache``
    (perplexity_eval.py:693-745).  Returns the model."""
    num_kv_heads = model.config.num_key_value_heads
    G = model.config.num_attention_heads // num_kv_heads
    layers = model.model.layers
    patched = 0
    for idx, layer in enumerate(layers):
        if idx < min_layer:
            continue
        attn = layer.self_attn
        original = attn.forward

        def make(orig, layer_idx):
            def patched_forward(*args, **kwargs):
                def intercept(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                              enable_gqa=False):
                    return orthocache.orthocache_attention(query, key, value, num_query_groups=G, layer=layer_idx)
                old = F.scaled_dot_product_attention
                F.scaled_dot_product_attention = intercept
                try:
                    return orig(*args, **kwargs)
                finally:
                    F.scaled_dot_product_attention = old
            return patched_forward

        attn.forward = make(original, idx)
        patched += 1
    if orthocache.verbose:
        print(f"  Patched {patched}/{len(layers)} layers (G={G}, layers {min_layer}-{len(layers) - 1})")
    return model
