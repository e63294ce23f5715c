"""GPU test of the allocation-free entry point oc_fused_attention_v2_noalloc.

Callers that cannot allocate device memory (a plugin that only receives its
inputs and outputs, code running inside another framework's memory pool)
use this entry point; it keeps its scratch in an array the library reserves
statically.  The test calls it through the C ABI twice in a row, on
different inputs, and checks each result against oc_fused_attention_v2 with
a caller-provided workspace, within the float16 tolerance of the parity tests.
It lives in its own file, collected last, and also passes when run alone.
"""

import pytest
import torch

from orthocache_gpu_b200 import _lib
from orthocache_gpu_b200.synthetic import mha_inputs

pytestmark = pytest.mark.gpu

TOL = 2e-3  # float16 output tolerance (max abs), as in the parity tests


def _call(lib, fn, q, k, v, out, mask, ctrl, zeta, extra):
    return fn(q.data_ptr(), _lib.OC_F16, q.stride(0),
              k.data_ptr(), _lib.OC_F16, k.stride(0), k.stride(1),
              v.data_ptr(), _lib.OC_F16, v.stride(0), v.stride(1),
              q.shape[0], k.shape[1], q.shape[1], zeta, 0, 0,
              out.data_ptr(), _lib.OC_F16, out.stride(0),
              mask.data_ptr(), ctrl.data_ptr(), ctrl[1:].data_ptr(), *extra,
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_entry_point_matches_workspace_entry_point():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    for seed, (heads, seq) in enumerate([(8, 4096), (32, 2048)]):
        x = mha_inputs(heads, seq, 128, seed=100 + seed)
        q, k, v = (t.to(dev) for t in x.torch(torch.float16))
        tiles = seq // 64
        ref = torch.empty(heads, 128, dtype=torch.float16, device=dev)
        got = torch.full_like(ref, float("nan"))
        mref = torch.empty(heads, tiles, dtype=torch.uint8, device=dev)
        mgot = torch.empty_like(mref)
        cref = torch.zeros(2, dtype=torch.int32, device=dev)
        cgot = torch.zeros(2, dtype=torch.int32, device=dev)
        splits = lib.oc_auto_num_splits(tiles, torch.cuda.get_device_properties(dev).multi_processor_count)
        ws = torch.zeros(lib.oc_workspace_bytes(heads, 1, tiles, 128), dtype=torch.uint8, device=dev)
        assert _call(lib, lib.oc_fused_attention_v2, q, k, v, ref, mref, cref, 1.0,
                     (ws.data_ptr(), ws.numel())) == 0
        assert _call(lib, lib.oc_fused_attention_v2_noalloc, q, k, v, got, mgot, cgot, 1.0, ()) == 0
        torch.cuda.synchronize()
        assert cgot[1].item() == 0 and cref[1].item() == 0, "device status word set"
        assert cgot[0].item() == cref[0].item()
        assert torch.equal(mgot, mref)
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= TOL, f"call {seed}: max abs error {err}"


def test_noalloc_rejects_problems_beyond_its_scratch():
    # head_dim 256 needs about 2.8 MiB of split-K scratch, more than the 2 MiB
    # reserved array: refused before any memory is touched
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    q = torch.zeros(2, 256, dtype=torch.float16, device=dev)
    out = torch.empty_like(q)
    ctrl = torch.zeros(2, dtype=torch.int32, device=dev)
    seq = 64 * 16
    rc = lib.oc_fused_attention_v2_noalloc(
        q.data_ptr(), _lib.OC_F16, 256, 16, _lib.OC_F16, seq * 256, 256, 16, _lib.OC_F16, seq * 256, 256,
        2, seq, 256, 1.0, 0, 148, out.data_ptr(), _lib.OC_F16, 256, None, None,
        ctrl[1:].data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 5
    assert "2 MiB" in lib.oc_status_string(rc).decode()
