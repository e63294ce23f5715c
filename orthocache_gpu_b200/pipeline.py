"""``orthocache_forward``: the reference pipeline entry point, fused mode on B200.

Drop-in for ``orthocache_gpu.pipeline.orthocache_forward``
(j-arndt/orthocache-gpu, src/orthocache_gpu/pipeline.py:312-456) for the
decode modes on the hot path:

* ``mode='triton_fused'`` runs the library's fused ζ-gated split-K kernel
  (the name is kept for compatibility; there is no Triton).  Keys / values
  in the pipeline's (seq, heads, head_dim) layout are streamed in place
  through their strides: no per-call permute + contiguous copy of the cache
  (pipeline.py:438-439);
* ``mode='dense'`` is the reference's dense einsum/softmax baseline
  (pipeline.py:558-568), in PyTorch;
* ``mode='compact'`` is the 512-token block path: a two-gate block mask
  (logit bound and ζ over 512-point Walsh bands) computed with PyTorch ops,
  then one kernel launch attending only to the retained blocks
  (``orthocache_gpu_b200.compact``).

Like the reference, the fused mode decodes the first query token only and
returns (1, num_heads, head_dim).  Its ``eviction_rate`` is the measured rate
(the reference's GPU path always reports 0.0, pipeline.py:451).
"""

from __future__ import annotations

import dataclasses
import enum
import time

import torch
import torch.nn.functional as F

from .fused_eviction import fused_orthocache_attention_v2


class BypassFlag(enum.IntFlag):
    """Dispatch flags (pipeline.py:62-74)."""
    NONE = 0
    CROSSOVER_BYPASS = 1 << 0
    DENSE_EXPLICIT = 1 << 1
    TRITON_FUSED = 1 << 2
    SPECTRAL_EVICTION = 1 << 3
    ZERO_ACTIVE = 1 << 4
    TAU_AUTO = 1 << 5
    PERFECT_EVICTION = 1 << 6
    HW_AUTO_DETECTED = 1 << 7


class TelemetryLevel(enum.IntEnum):
    """Metadata verbosity (pipeline.py:77-87)."""
    SILENT = 0
    FLAGS = 1
    VERBOSE = 2


def format_bypass_reason(flags: BypassFlag, seq_len_k: int = 0, threshold: int = 0, profile=None) -> str:
    """Human-readable form of ``flags`` (pipeline.py:90-117); never on the hot path."""
    parts = []
    if flags & BypassFlag.CROSSOVER_BYPASS:
        p = f"seq_len_k={seq_len_k} < crossover={threshold}"
        if profile:
            p += f" on {profile.name} ({profile.sm_count} SMs, {profile.mem_bandwidth_gbps:.0f} GB/s)"
        parts.append(p)
    if flags & BypassFlag.DENSE_EXPLICIT:
        parts.append("mode=dense (explicit)")
    if flags & BypassFlag.TRITON_FUSED:
        parts.append("mode=triton_fused (fused CUDA kernel)")
    if flags & BypassFlag.ZERO_ACTIVE:
        parts.append("all blocks evicted")
    if flags & BypassFlag.HW_AUTO_DETECTED:
        parts.append("GPU auto-detected")
    return "; ".join(parts) if parts else "no flags set"


@dataclasses.dataclass(frozen=True)
class GPUProfile:
    """Hardware profile (pipeline.py:121-203).  The B200 entry holds this
    pool's measured figures (148 SMs, measured copy bandwidth)."""
    name: str
    sm_count: int
    mem_bandwidth_gbps: float
    sram_per_sm_kb: int
    crossover_seq_len: int
    compute_class: str = "datacenter"


# crossover 512 as the reference's B200 entry (pipeline.py:192-196): below one
# 512-token block the compact mode runs dense
B200_PROFILE = GPUProfile(name="B200", sm_count=148, mem_bandwidth_gbps=6456.0, sram_per_sm_kb=228,
                          crossover_seq_len=512, compute_class="hpc")


def get_hardware_profile(device: torch.device | None = None) -> GPUProfile:
    if device is not None and device.type == "cuda":
        props = torch.cuda.get_device_properties(device)
        if "B200" in props.name:
            return B200_PROFILE
        return GPUProfile(name=f"{props.name} (auto-detected)", sm_count=props.multi_processor_count,
                          mem_bandwidth_gbps=0.0, sram_per_sm_kb=0, crossover_seq_len=0, compute_class="unknown")
    return B200_PROFILE


def _dense_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Dense attention baseline (pipeline.py:558-568)."""
    scale = torch.sqrt(torch.tensor(head_dim, dtype=torch.float32, device=q.device))
    logits = torch.einsum("qhd,khd->qkh", q, keys) / scale
    weights = F.softmax(logits, dim=1)
    return torch.einsum("qkh,khd->qhd", weights, values)


def orthocache_forward(
    q: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    block_size: int = 512,
    zeta_max: float = 5.0,
    tau: float | None = None,
    mode: str = "compact",
    crossover_threshold: int = 0,
    telemetry: TelemetryLevel = TelemetryLevel.FLAGS,
) -> tuple[torch.Tensor, dict]:
    """Pipeline entry point (pipeline.py:312-456).

    q (seq_len_q, num_heads, head_dim); keys / values (seq_len_k, num_heads,
    head_dim).  See the module docstring for the supported modes.
    """
    seq_len_k, num_heads, head_dim = keys.shape
    seq_len_q = q.shape[0]
    num_blocks = seq_len_k // block_size

    crossover_fallback = False
    original_mode = mode
    if seq_len_k < crossover_threshold and mode in ("compact", "triton_fused"):
        mode = "dense"
        crossover_fallback = True

    if telemetry == TelemetryLevel.SILENT:
        metadata: dict = {}
    else:
        metadata = {
            "mode": original_mode, "actual_mode": mode, "crossover_fallback": crossover_fallback,
            "crossover_threshold": crossover_threshold, "seq_len_q": seq_len_q, "seq_len_k": seq_len_k,
            "num_blocks": num_blocks, "num_heads": num_heads, "head_dim": head_dim,
            "block_size": block_size, "zeta_max": zeta_max,
        }

    if mode == "dense":
        t0 = time.perf_counter()
        output = _dense_attention(q, keys, values, head_dim)
        if telemetry != TelemetryLevel.SILENT:
            metadata["latency_ms"] = (time.perf_counter() - t0) * 1000
            metadata["eviction_rate"] = 0.0
        return output, metadata

    if mode == "triton_fused":
        t0 = time.perf_counter()
        q_heads = q[0]                              # (num_heads, head_dim): first query token
        k_heads = keys.permute(1, 0, 2)             # strided view, no copy
        v_heads = values.permute(1, 0, 2)
        want_stats = telemetry != TelemetryLevel.SILENT
        out_heads, fused_meta = fused_orthocache_attention_v2(q_heads, k_heads, v_heads, zeta_max=zeta_max,
                                                              stats=want_stats)
        output = out_heads.unsqueeze(0)
        if want_stats:
            tile_size = 64
            metadata["latency_ms"] = (time.perf_counter() - t0) * 1000
            metadata["eviction_rate"] = fused_meta.get("eviction_rate", 0.0)
            metadata["tile_size_fused"] = tile_size
            metadata["num_tiles_fused"] = seq_len_k // tile_size
            metadata["num_splits"] = fused_meta.get("num_splits", 1)
            metadata["tile_assignment"] = "interleaved"
            if telemetry >= TelemetryLevel.FLAGS:
                flags = BypassFlag.TRITON_FUSED
                if fused_meta.get("tiles_retained", 1) == 0:
                    flags |= BypassFlag.ZERO_ACTIVE
                metadata["bypass_flags"] = int(flags)
        return output, metadata

    hw = get_hardware_profile(q.device)
    if seq_len_k < hw.crossover_seq_len:  # hardware-aware bypass (pipeline.py:397-421)
        t0 = time.perf_counter()
        output = _dense_attention(q, keys, values, head_dim)
        if telemetry >= TelemetryLevel.FLAGS:
            flags = BypassFlag.CROSSOVER_BYPASS
            if hw.compute_class == "unknown":
                flags |= BypassFlag.HW_AUTO_DETECTED
            metadata["latency_ms"] = (time.perf_counter() - t0) * 1000
            metadata["eviction_rate"] = 0.0
            metadata["bypass_flags"] = int(flags)
            metadata["crossover_threshold"] = hw.crossover_seq_len
            metadata["gpu_profile"] = hw.name
            if telemetry >= TelemetryLevel.VERBOSE:
                metadata["crossover_reason"] = format_bypass_reason(flags, seq_len_k, hw.crossover_seq_len, hw)
        return output, metadata

    if mode == "compact":
        from .compact import compact_forward
        output, meta = compact_forward(q, keys, values, block_size, zeta_max, tau, {})
        if telemetry != TelemetryLevel.SILENT:
            metadata.update(meta)
        return output, metadata

    raise ValueError(f"Unknown mode: {mode!r}. Use 'dense', 'compact', or 'triton_fused'.")
