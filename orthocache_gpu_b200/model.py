"""A Llama-shaped decoder whose decode attention is the fused eviction kernel.

The reference evaluates its gate inside HF Llama decoding (TinyLlama-1.1B,
eval/perplexity_eval.py:693-745).  This module is the self-contained
equivalent for measurement: random-initialised weights of the
TinyLlama-1.1B shape (22 layers, hidden 2048, 32 query / 4 kv heads,
head_dim 64, MLP 5632, vocab 32000, RMSNorm, rotary embeddings), a
preallocated KV cache, dense causal prefill, and greedy decoding in which
every layer's attention runs the Cauchy-Schwarz-gated kernel over the
cache's whole 64-token tiles.  Tokens after the last whole tile (fewer than
64) are attended densely and merged with the kernel's softmax state by the
library's log-sum-exp merge, so nothing is dropped except evicted tiles.
No pretrained weights are loaded (none are needed to measure the path).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from . import _lib
from .distributed import merge_states, shard_partials

LOG2E = 1.4426950408889634


@dataclass
class LlamaShape:
    layers: int = 22
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 64
    mlp: int = 5632
    vocab: int = 32000
    rope_theta: float = 10000.0
    eps: float = 1e-5


def _rms(x, w, eps):
    return (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def _rope_tables(max_len, hd, theta, device):
    """cos / sin tables (max_len, hd) of the rotate-half rotary embedding (same values as _rope)."""
    pos = torch.arange(max_len, device=device)
    inv = theta ** (-torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd)
    ang = pos.float()[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.cos()], -1), torch.cat([ang.sin(), ang.sin()], -1)


def _rope_t(x, cos, sin):
    """Rotary embedding of x (..., T, hd) with the table rows of its positions."""
    hd = x.shape[-1]
    rot = torch.cat([-x[..., hd // 2:], x[..., : hd // 2]], -1)
    return (x.float() * cos + rot.float() * sin).to(x.dtype)


class GatedLlama:
    """Random-initialised Llama-shaped decoder with a preallocated KV cache.

    ``tau``: a float (the Cauchy-Schwarz threshold of every layer), or
    "median" to calibrate each layer's threshold at the first decode step as
    the median per-tile bound max_g |q_g| |K_high|_F (about half the tiles
    evicted), None for dense decode attention with torch SDPA, or "flash"
    for dense flash-decoding (flashinfer) of every cached token.
    """

    def __init__(self, shape: LlamaShape, max_len: int, device="cuda", dtype=torch.bfloat16, seed: int = 0):
        self.s, self.dev, self.dtype, self.max_len = shape, torch.device(device), dtype, max_len
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)

        def w(*shape_, std=0.02):
            return (torch.randn(*shape_, generator=g, device=self.dev) * std).to(dtype)

        s = shape
        ones = lambda n: torch.ones(n, device=self.dev, dtype=dtype)  # noqa: E731
        self.embed = w(s.vocab, s.hidden)
        self.layers = [dict(ln1=ones(s.hidden), wq=w(s.hidden, s.heads * s.head_dim),
                            wk=w(s.hidden, s.kv_heads * s.head_dim), wv=w(s.hidden, s.kv_heads * s.head_dim),
                            wo=w(s.heads * s.head_dim, s.hidden), ln2=ones(s.hidden),
                            w1=w(s.hidden, s.mlp), w3=w(s.hidden, s.mlp), w2=w(s.mlp, s.hidden))
                       for _ in range(s.layers)]
        # weights in the (out_features, in_features) layout of a linear layer (each output a
        # contiguous row); one GEMV each for q|k|v and for the two MLP inputs (the same weights,
        # concatenated; w1 | w3 rows interleaved, row 2j = w1's output j and row 2j + 1 = w3's,
        # the layout of oc_gemv's SILU_MUL epilogue)
        for L in self.layers:
            L["wqkv"] = torch.cat([L.pop("wq"), L.pop("wk"), L.pop("wv")], 1).t().contiguous()
            w1, w3 = L.pop("w1"), L.pop("w3")
            L["w13"] = torch.stack([w1.t(), w3.t()], 1).reshape(2 * s.mlp, s.hidden).contiguous()
            L["wo"] = L["wo"].t().contiguous()
            L["w2"] = L["w2"].t().contiguous()
        self.norm = ones(s.hidden)
        self.lm_head = w(s.hidden, s.vocab).t().contiguous()
        # token-major caches (max_len, kv_heads, head_dim): a prefix [:n] is contiguous (what dense
        # flash-decoding wants); the fused kernel reads the (kv_heads, n, head_dim) view through its strides
        self.k_cache = [torch.zeros(max_len, s.kv_heads, s.head_dim, device=self.dev, dtype=dtype)
                        for _ in range(s.layers)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self._cos, self._sin = _rope_tables(max_len, s.head_dim, s.rope_theta, self.dev)
        self.length = 0
        self.tau: List[Optional[float]] = [None] * s.layers
        self.kept = 0
        self.tiles = 0

    def weight_bytes(self) -> int:
        """Bytes of the weights one decode step reads (all layers, final norm, LM head; not the embedding)."""
        n = sum(t.numel() * t.element_size() for L in self.layers for t in L.values())
        return n + self.norm.numel() * self.norm.element_size() + self.lm_head.numel() * self.lm_head.element_size()

    # ---------------------------------------------------------------- blocks
    def _qkv(self, L, h, pos):
        s = self.s
        T = h.shape[0]
        qkv = F.linear(h, L["wqkv"])
        nq, nk = s.heads * s.head_dim, s.kv_heads * s.head_dim
        q = qkv[:, :nq].view(T, s.heads, s.head_dim).transpose(0, 1)
        k = qkv[:, nq:nq + nk].view(T, s.kv_heads, s.head_dim).transpose(0, 1)
        v = qkv[:, nq + nk:].view(T, s.kv_heads, s.head_dim).transpose(0, 1)
        cos, sin = self._cos.index_select(0, pos), self._sin.index_select(0, pos)   # (T, hd) tables
        return _rope_t(q, cos, sin), _rope_t(k, cos, sin), v

    def _mlp(self, L, x):
        h = _rms(x, L["ln2"], self.s.eps)
        ab = F.linear(h, L["w13"]).view(*h.shape[:-1], -1, 2)
        return x + F.linear(F.silu(ab[..., 0]) * ab[..., 1], L["w2"])

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """Dense causal attention over the prompt; fills the cache; returns last-position logits."""
        s = self.s
        T = tokens.shape[0]
        pos = torch.arange(T, device=self.dev)
        x = self.embed[tokens]
        for i, L in enumerate(self.layers):
            q, k, v = self._qkv(L, _rms(x, L["ln1"], s.eps), pos)
            self.k_cache[i][:T] = k.transpose(0, 1)
            self.v_cache[i][:T] = v.transpose(0, 1)
            a = F.scaled_dot_product_attention(q[None], k[None], v[None], is_causal=True, enable_gqa=True)[0]
            x = x + F.linear(a.transpose(0, 1).reshape(T, -1), L["wo"])
            x = self._mlp(L, x)
        self.length = T
        return F.linear(_rms(x[-1:], self.norm, s.eps), self.lm_head)

    # ---------------------------------------------------------------- decode
    def _median_bound(self, q, k_tiles):
        """Median over (kv head, tile) of max_g |q_g| * |K_high|_F (the gate's bound, in torch)."""
        s = self.s
        G = s.heads // s.kv_heads
        kt = k_tiles.float().view(s.kv_heads, -1, 64, s.head_dim)
        e_high = 0.5 * (kt[:, :, :32] - kt[:, :, 32:]).pow(2).sum((-1, -2))      # (KVH, T)
        qn = q.float().view(s.kv_heads, G, s.head_dim).norm(dim=-1).amax(-1)      # (KVH,)
        return float((qn[:, None] * e_high.sqrt()).median())

    def _attend(self, i, q, tau_mode):
        """Decode attention of layer i for q (Hq, hd) over the cache [0, length)."""
        s = self.s
        G = s.heads // s.kv_heads
        n = self.length
        full = n - n % 64
        kc, vc = self.k_cache[i].transpose(0, 1), self.v_cache[i].transpose(0, 1)  # (kv_heads, max_len, hd) views
        scale = LOG2E / math.sqrt(s.head_dim)
        if tau_mode == "flash":  # dense flash-decoding of every cached token (the fair dense arm)
            import flashinfer
            return flashinfer.single_decode_with_kv_cache(q, self.k_cache[i][:n], self.v_cache[i][:n], kv_layout="NHD")
        if tau_mode is None or full == 0:  # dense (reference point, or no whole tile yet)
            a = F.scaled_dot_product_attention(q[None, :, None], kc[None, :, :n], vc[None, :, :n], enable_gqa=True)
            return a[0, :, 0]
        if self.tau[i] is None:
            self.tau[i] = self._median_bound(q, kc[:, :full]) if tau_mode == "median" else float(tau_mode)
        m, l, acc, _ = shard_partials(q, kc[:, :full], vc[:, :full], self.tau[i], G, stats=False)
        ms, ls, accs = [m], [l], [acc]
        if n > full:  # ragged tail: dense, as a second softmax state in log2 units
            kt = kc[:, full:n].repeat_interleave(G, 0).float()
            vt = vc[:, full:n].repeat_interleave(G, 0).float()
            sc = (kt @ q.float()[:, :, None])[..., 0] * scale            # (Hq, r)
            mt = sc.amax(-1)
            pt = torch.exp2(sc - mt[:, None])
            ms.append(mt)
            ls.append(pt.sum(-1))
            accs.append((pt[:, None, :] @ vt)[:, 0])
        return merge_states(torch.stack(ms, 1).contiguous(), torch.stack(ls, 1).contiguous(),
                            torch.stack(accs, 1).contiguous(), self.dtype)

    @torch.no_grad()
    def step(self, token: torch.Tensor, tau_mode) -> torch.Tensor:
        """One decode step for a (1,) token; returns logits (1, vocab)."""
        s = self.s
        pos = torch.full((1,), self.length, device=self.dev, dtype=torch.long)
        x = self.embed[token]
        for i, L in enumerate(self.layers):
            q, k, v = self._qkv(L, _rms(x, L["ln1"], s.eps), pos)
            self.k_cache[i][self.length] = k[:, 0]
            self.v_cache[i][self.length] = v[:, 0]
            self.length += 1
            a = self._attend(i, q[:, 0].contiguous(), tau_mode)
            self.length -= 1
            x = x + F.linear(a.reshape(1, -1), L["wo"])
            x = self._mlp(L, x)
        self.length += 1
        return F.linear(_rms(x, self.norm, s.eps), self.lm_head)

    # ---------------------------------------------------------------- CUDA-graph decode
    @torch.no_grad()
    def _step_dev(self, tok, npos, dense_window: Optional[int] = None):
        """One decode step from device state: tok (1,) next token, npos (1,) cache length;
        both are updated in place (argmax token, length + 1).

        Seven launches per layer: the q|k|v GEMV with the residual add + RMSNorm
        in its prologue and rotary embedding + cache append in its epilogue;
        the fused decode attention over whole tiles (+ its merge) and the
        ragged-tail merge; the output projection; the MLP input GEMV (residual
        add + RMSNorm prologue, silu(a) * b epilogue); the MLP output
        projection.  Same arithmetic as ``step`` up to fp32 summation order.
        ``dense_window``: timing arm only -- dense flash-decoding (flashinfer)
        of the first ``dense_window`` cached tokens instead of the fused
        kernel (a CUDA graph needs a fixed length for it)."""
        s = self.s
        lib, dev = _lib.load(), self.dev
        st, dt = _lib.stream_ptr(dev), _lib.dtype_code(self.embed)
        G = s.heads // s.kv_heads
        res = [self.embed[tok].contiguous(), torch.empty((1, s.hidden), device=dev, dtype=self.dtype)]
        q = torch.empty((s.heads, s.head_dim), device=dev, dtype=self.dtype)
        a = torch.empty_like(q)
        o = torch.empty((1, s.hidden), device=dev, dtype=self.dtype)
        g = torch.empty((1, s.mlp), device=dev, dtype=self.dtype)
        y = torch.empty((1, s.hidden), device=dev, dtype=self.dtype)
        full_dev = (torch.div(npos + 1, 64, rounding_mode="floor") * 64).to(torch.int32)
        cap = self.max_len - self.max_len % 64
        tok_stride = s.kv_heads * s.head_dim
        cur, prev_y = 0, None
        for i, L in enumerate(self.layers):
            _lib.check(lib.oc_gemv_qkv_rope(
                res[cur].data_ptr(), _lib.ptr(prev_y), L["ln1"].data_ptr(), s.eps, res[1 - cur].data_ptr(),
                L["wqkv"].data_ptr(), L["wqkv"].stride(0), s.hidden, s.heads, s.kv_heads, s.head_dim,
                self._cos.data_ptr(), self._sin.data_ptr(), npos.data_ptr(), q.data_ptr(),
                self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr(), tok_stride, dt, st),
                "oc_gemv_qkv_rope")
            cur = 1 - cur
            if dense_window is not None:
                import flashinfer
                a = flashinfer.single_decode_with_kv_cache(q, self.k_cache[i][:dense_window],
                                                           self.v_cache[i][:dense_window], kv_layout="NHD")
            else:
                kc, vc = self.k_cache[i].transpose(0, 1), self.v_cache[i].transpose(0, 1)
                m, l, acc, _ = shard_partials(q, kc[:, :cap], vc[:, :cap], self.tau[i], G, stats=False,
                                              seq_len_dev=full_dev)
                _lib.check(lib.oc_tail_merge(q.data_ptr(), s.heads, s.kv_heads, s.head_dim,
                                             self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr(), tok_stride,
                                             self.max_len, npos.data_ptr(), m.data_ptr(), l.data_ptr(),
                                             acc.data_ptr(), LOG2E / math.sqrt(s.head_dim), a.data_ptr(), dt, st),
                           "oc_tail_merge")
            _lib.check(lib.oc_gemv(a.data_ptr(), 0, 0, 0.0, 0, L["wo"].data_ptr(), L["wo"].stride(0),
                                   s.heads * s.head_dim, s.hidden, o.data_ptr(), 0, dt, st), "oc_gemv")
            _lib.check(lib.oc_gemv(res[cur].data_ptr(), o.data_ptr(), L["ln2"].data_ptr(), s.eps,
                                   res[1 - cur].data_ptr(), L["w13"].data_ptr(), L["w13"].stride(0), s.hidden,
                                   2 * s.mlp, g.data_ptr(), 1, dt, st), "oc_gemv")
            cur = 1 - cur
            _lib.check(lib.oc_gemv(g.data_ptr(), 0, 0, 0.0, 0, L["w2"].data_ptr(), L["w2"].stride(0), s.mlp,
                                   s.hidden, y.data_ptr(), 0, dt, st), "oc_gemv")
            prev_y = y
        logits = torch.empty((1, s.vocab), device=dev, dtype=self.dtype)
        _lib.check(lib.oc_gemv(res[cur].data_ptr(), y.data_ptr(), self.norm.data_ptr(), s.eps, 0,
                               self.lm_head.data_ptr(), self.lm_head.stride(0), s.hidden, s.vocab,
                               logits.data_ptr(), 0, dt, st), "oc_gemv")
        tok.copy_(logits.argmax(-1))
        npos.add_(1)
        return logits

    @torch.no_grad()
    def generate_graph(self, prompt: torch.Tensor, steps: int, tau_mode="median", dense: bool = False,
                       profile_replay: Optional[int] = None) -> Dict:
        """Greedy decoding with each decode step replayed from one captured CUDA graph.

        Prefill and the first step run eagerly (the first step calibrates each
        layer's tau); the step is then captured once and replayed ``steps - 1``
        times, with lengths and tokens kept on the device (no host sync per token).
        Returns the per-step device time (CUDA events around the replays).
        ``dense=True`` times the dense arm: the same step with flashinfer
        decoding over the prompt's tokens (a fixed window) in place of the
        fused kernel; its tokens are not a faithful greedy continuation.
        """
        self.length = 0
        self.tau = [None] * self.s.layers
        logits = self.prefill(prompt)
        tok = logits.argmax(-1)
        first = self.step(tok, "flash" if dense else tau_mode)   # eager: sets self.tau
        window = prompt.shape[0] if dense else None
        tok_d = first.argmax(-1).reshape(1).clone()
        npos = torch.full((1,), self.length, dtype=torch.long, device=self.dev)
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            # a warm-up step outside the capture (workspaces, tensor maps), undone afterwards
            t0, n0 = tok_d.clone(), npos.clone()
            self._step_dev(tok_d, npos, window)
            tok_d.copy_(t0)
            npos.copy_(n0)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=st):
                self._step_dev(tok_d, npos, window)
        torch.cuda.current_stream().wait_stream(st)
        toks = [int(tok), int(tok_d)]
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        hist = []
        for i in range(steps - 1):
            if i == profile_replay:
                torch.cuda.cudart().cudaProfilerStart()
            g.replay()
            if i == profile_replay:
                torch.cuda.cudart().cudaProfilerStop()
            hist.append(tok_d.clone())
        b.record()
        torch.cuda.synchronize()
        toks += [int(t) for t in hist]
        self.length = int(npos)
        ms = a.elapsed_time(b) / max(1, steps - 1)
        return {"tokens": toks, "ms_per_token": ms, "tau": self.tau, "final_length": self.length}

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, steps: int, tau_mode="median") -> Dict:
        """Greedy decoding: prefill, then ``steps`` decode steps; per-step device time."""
        self.length = 0
        self.tau = [None] * self.s.layers
        logits = self.prefill(prompt)
        tok = logits.argmax(-1)
        out, times = [int(tok)], []
        for _ in range(steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            logits = self.step(tok, tau_mode)
            tok = logits.argmax(-1)
            b.record()
            out.append(tok)
            times.append((a, b))
        torch.cuda.synchronize()
        ms = [x.elapsed_time(y) for x, y in times]
        return {"tokens": [int(t) for t in out], "ms_per_token": sorted(ms)[len(ms) // 2],
                "ms_mean": sum(ms) / len(ms), "tau": self.tau, "final_length": self.length}
