"""CPU tests of the host layer: assertion messages, C-ABI exports, no CPU fallback."""

import ctypes
import os
import re

import pytest
import torch

import orthocache_gpu_b200 as oc
from orthocache_gpu_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "orthocache_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const char\*|int|size_t|void)\s+(oc_\w+)\(", src, re.M)))


def test_header_declares_the_reference_entry_points():
    names = declared_symbols()
    for n in ["oc_fwht_eviction", "oc_fused_attention_v1", "oc_fused_attention_v2",
              "oc_fused_attention_v3_gqa", "oc_fused_attention_paged", "oc_lse_merge"]:
        assert n in names


@pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="library not built")
def test_library_loads_and_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    # every binding signature names a declared symbol
    assert set(_lib.SIGNATURES) <= set(declared_symbols())
    l = _lib.load()
    assert l.oc_version() >= 100
    assert l.oc_auto_num_splits(512, 148) == 128      # the reference heuristic
    assert l.oc_auto_num_splits(16, 148) == 4
    assert l.oc_auto_num_splits(0, 148) == 1
    assert l.oc_auto_num_splits(10000, 148) == 148
    # tickets + two partial states (acc, m, l) per team of warps; no per-tile scratch
    ws = l.oc_workspace_bytes(32, 1, 512, 128)
    assert ws >= 2 * 1280 * (128 + 4) * 4
    assert ws == l.oc_workspace_bytes(4096, 1, 1 << 20, 128)
    assert l.oc_workspace_bytes(32, 8, 512, 128) > ws
    assert l.oc_status_string(3).decode().startswith("workspace")


@pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="library not built")
def test_c_abi_rejects_bad_arguments_without_a_gpu():
    l = _lib.load()
    # null pointers / bad sizes are rejected before any CUDA call
    assert l.oc_fwht_eviction(None, 1, 128, 128, 128, 5.0, None, None, None, None) == 1
    assert l.oc_lse_merge(None, None, None, 1, 1, 128, None, 0, None) == 1
    # unsupported head_dim
    buf = ctypes.create_string_buffer(64 * 1024 + 16)
    addr = (ctypes.addressof(buf) + 15) & ~15
    st = ctypes.c_uint32(0)
    assert l.oc_fwht_eviction(addr, 1, 64, 100, 100, 5.0, addr, None, ctypes.addressof(st), None) == 2
    # model-step GEMV: null input, K not a multiple of 8, odd N, K beyond the prologue limit, odd head_dim
    assert l.oc_gemv(None, None, None, 1e-5, None, addr, 64, 64, 64, addr, 0, 2, None) == 1
    assert l.oc_gemv(addr, None, None, 1e-5, None, addr, 64, 60, 64, addr, 0, 2, None) == 1
    assert l.oc_gemv(addr, None, None, 1e-5, None, addr, 64, 64, 63, addr, 0, 2, None) == 1
    assert l.oc_gemv(addr, None, addr, 1e-5, None, addr, 16384, 16384, 64, addr, 0, 2, None) == 1
    assert l.oc_gemv(addr, None, None, 1e-5, None, addr, 64, 64, 64, addr, 7, 2, None) == 1   # epilogue
    assert l.oc_gemv(addr, None, addr, 1e-5, addr, addr, 64, 64, 64, addr, 0, 2, None) == 1  # x_out aliases x
    assert l.oc_gemv_qkv_rope(addr, None, addr, 1e-5, None, addr, 64, 64, 8, 2, 63, addr, addr, addr, addr, addr,
                              addr, 256, 2, None) == 1


def _t(*shape):
    return torch.randn(*shape)


def test_v1_assertions_match_reference_messages():
    q, k, v = _t(1, 128), _t(256, 128), _t(256, 128)
    with pytest.raises(AssertionError, match="head_dim.*must be a power of 2"):
        oc.fused_orthocache_attention(_t(1, 100), _t(256, 100), _t(256, 100), zeta_max=5.0)
    with pytest.raises(AssertionError, match="tile_size.*must be a power of 2"):
        oc.fused_orthocache_attention(q, k, v, zeta_max=5.0, tile_size=50)
    with pytest.raises(AssertionError, match="not divisible by tile_size"):
        oc.fused_orthocache_attention(q, _t(250, 128), _t(250, 128), zeta_max=5.0)
    with pytest.raises(AssertionError, match=r"q must be \(1, head_dim\)"):
        oc.fused_orthocache_attention(_t(2, 128), k, v, zeta_max=5.0)


def test_v2_v3_paged_assertions_match_reference_messages():
    with pytest.raises(AssertionError, match="num_splits.*greater than 0"):
        oc.fused_orthocache_attention_v2(_t(2, 64), _t(2, 128, 64), _t(2, 128, 64), 5.0, num_splits=0)
    with pytest.raises(AssertionError, match="not divisible by tile_size"):
        oc.fused_orthocache_attention_v2(_t(2, 64), _t(2, 100, 64), _t(2, 100, 64), 5.0)
    with pytest.raises(AssertionError, match="num_query_heads"):
        oc.fused_orthocache_attention_v3_gqa(_t(6, 64), _t(2, 128, 64), _t(2, 128, 64), 1.0, num_query_groups=4)
    bt = torch.tensor([[0, 1]], dtype=torch.int32)
    with pytest.raises(AssertionError, match="head_dim.*power of 2"):
        oc.fused_orthocache_attention_paged(_t(1, 2, 63), _t(4, 2, 32, 63), _t(4, 2, 32, 63), bt, zeta_max=5.0)
    with pytest.raises(AssertionError, match="block_size.*power of 2"):
        oc.fused_orthocache_attention_paged(_t(1, 2, 64), _t(4, 2, 31, 64), _t(4, 2, 31, 64), bt, zeta_max=5.0)


def test_no_cpu_fallback():
    q, k, v = _t(1, 128), _t(256, 128), _t(256, 128)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        oc.fused_orthocache_attention(q, k, v, zeta_max=5.0)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        oc.fused_orthocache_attention_v2(_t(2, 128), _t(2, 256, 128), _t(2, 256, 128), 5.0)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        oc.triton_fwht_eviction(k, 5.0)


def test_other_tile_sizes_are_refused_clearly():
    with pytest.raises(NotImplementedError, match="64-token tile"):
        oc.fused_orthocache_attention_v2(_t(2, 64), _t(2, 128, 64), _t(2, 128, 64), 5.0, tile_size=32)


def test_walsh_matrix_matches_oracle():
    from oracle import orthocache_oracle as orc
    import numpy as np
    for n in (8, 64):
        np.testing.assert_array_equal(oc.generate_walsh_matrix(n).numpy(), orc.walsh_matrix(n))


def test_pipeline_dense_mode_and_compact_crossover_bypass_run_on_cpu():
    q, k, v = _t(1, 4, 64), _t(256, 4, 64), _t(256, 4, 64)
    out, meta = oc.orthocache_forward(q, k, v, mode="dense")
    assert out.shape == (1, 4, 64) and meta["actual_mode"] == "dense" and meta["eviction_rate"] == 0.0
    # shorter than the B200 crossover (512): compact mode attends densely and says so
    out2, meta2 = oc.orthocache_forward(q, k, v, mode="compact", telemetry=oc.TelemetryLevel.VERBOSE)
    assert torch.equal(out, out2) and meta2["bypass_flags"] & oc.BypassFlag.CROSSOVER_BYPASS
    assert "crossover=512" in meta2["crossover_reason"]
    with pytest.raises(ValueError, match="Unknown mode"):
        oc.orthocache_forward(q, _t(1024, 4, 64), _t(1024, 4, 64), mode="bogus")


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(_lib.LIB_PATH), "oc_torch.so")),
                    reason="binding not built")
def test_compiled_binding_loads_and_exports_the_hot_calls():
    b = _lib.binding()
    assert b is not None and hasattr(b, "v2") and hasattr(b, "v3")
