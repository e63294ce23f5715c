"""ctypes binding of ``liborthocache_b200.so`` (the C ABI in include/orthocache_b200.h).

PyTorch provides device memory and the current CUDA stream; every compute
call goes through the C ABI.  There is no CPU fallback: a missing library or
a non-CUDA tensor raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "liborthocache_b200.so")

OC_F32, OC_F16, OC_BF16, OC_F8E4M3 = 0, 1, 2, 3
OC_GATE_ZETA, OC_GATE_CAUCHY_SCHWARZ = 0, 2
STATUS_BITS = {1: "a shared-memory pipeline wait timed out",
               2: "a block-table entry was outside [0, num_blocks)",
               4: "a seq_lens entry was negative, not a multiple of 64, or beyond the block table"}

_DTYPE = {torch.float32: OC_F32, torch.float16: OC_F16, torch.bfloat16: OC_BF16,
          torch.float8_e4m3fn: OC_F8E4M3}

_vp, _i, _i64, _d, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_double, C.c_size_t

SIGNATURES = {
    "oc_status_string": (C.c_char_p, [_i]),
    "oc_version": (_i, []),
    "oc_workspace_bytes": (_sz, [_i64, _i, _i64, _i]),
    "oc_auto_num_splits": (_i, [_i64, _i]),
    "oc_fwht_eviction": (_i, [_vp, _i, _i64, _i, _i64, _d, _vp, _vp, _vp, _vp]),
    "oc_fused_attention_v2": (_i, [_vp, _i, _i64, _vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i, _i64, _i, _d,
                                   _i, _i, _vp, _i, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "oc_fused_attention_v1": (_i, [_vp, _i, _vp, _i, _i64, _vp, _i, _i64, _i64, _i, _d, _i, _vp, _i, _vp, _vp,
                                   _vp, _vp, _sz, _vp]),
    "oc_fused_attention_v3_gqa": (_i, [_vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64,
                                       _i, _i, _i, _i64, _i, _d, _i, _i, _vp, _i, _i64, _i64, _vp, _vp, _vp, _vp,
                                       _sz, _vp]),
    "oc_fused_attention_paged": (_i, [_vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64,
                                      _i, _i, _vp, _i64, _i, _vp, _i, _i, _i, _i, _i, _d, _i, _i, _vp, _i, _i64,
                                      _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "oc_fused_attention_v2_noalloc": (_i, [_vp, _i, _i64, _vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i, _i64, _i,
                                           _d, _i, _i, _vp, _i, _i64, _vp, _vp, _vp, _vp]),
    "oc_lse_merge": (_i, [_vp, _vp, _vp, _i64, _i, _i, _vp, _i, _vp]),
    "oc_fused_attention_v3_shard": (_i, [_vp, _i, _i64, _vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i, _i, _i64,
                                         _i, _d, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
}

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Load the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"orthocache_gpu_b200: CUDA library not built ({LIB_PATH} missing); "
                        "run `python -m orthocache_gpu_b200._build` (needs nvcc)")
                lib = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, float16, bfloat16 "
                        "(or float8_e4m3fn for keys)") from None


def check(code: int, what: str) -> None:
    if code != 0:
        msg = load().oc_status_string(code).decode()
        raise RuntimeError(f"{what}: {msg} (code {code})")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("orthocache_gpu_b200 runs on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")
        if t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_sm_cache: dict = {}


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _sm_cache:
        _sm_cache[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _sm_cache[idx]


class _Workspace:
    """Zero-initialised split-K workspace and control words for one (device, stream)."""

    def __init__(self, device):
        self.device = device
        self.buf = torch.zeros(0, dtype=torch.uint8, device=device)
        # ctrl[0]: retained-tile counter, ctrl[1]: status bits
        self.ctrl = torch.zeros(2, dtype=torch.int32, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 2 * self.buf.numel()), dtype=torch.uint8, device=self.device)
        return self.buf

    def reset(self) -> None:
        self.buf.zero_()
        self.ctrl.zero_()


_ws: dict = {}


def workspace(device: torch.device) -> _Workspace:
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    w = _ws.get(key)
    if w is None:
        w = _ws[key] = _Workspace(device)
    return w


def read_stats(ws: _Workspace) -> int:
    """Synchronising read of the retained-tile counter; raises on a device status."""
    retained, status = ws.ctrl.tolist()
    if status:
        ws.reset()
        bits = [m for b, m in STATUS_BITS.items() if status & b]
        raise RuntimeError("orthocache_gpu_b200 kernel reported: " + "; ".join(bits))
    return int(retained)


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def prepare_kv(t: torch.Tensor) -> torch.Tensor:
    """A view whose last dim is contiguous and whose other strides and base are 16-byte aligned.

    Copies only when the given layout cannot be streamed directly.
    """
    es = t.element_size()
    ok = t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all((s * es) % 16 == 0 for s in t.stride()[:-1])
    if ok:
        return t
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def harmonize_kv(keys: torch.Tensor, values: torch.Tensor):
    """Keys and values in a dtype pair the kernels compile.

    float8 keys pair with any value dtype; otherwise keys and values must share
    a dtype, so a mixed pair is widened (exactly) to float32.
    """
    if keys.dtype == torch.float8_e4m3fn or keys.dtype == values.dtype:
        return keys, values
    return keys.float(), values.float()
