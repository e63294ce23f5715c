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
# ORTHOCACHE_B200_LIB selects another build of the same C ABI (e.g. a diagnostics build)
LIB_PATH = os.environ.get("ORTHOCACHE_B200_LIB") or os.path.join(_PKG, "_lib", "liborthocache_b200.so")

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
    "oc_debug_set_trace": (None, [_vp]),
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
                                      _i, _i, _vp, _i64, _i, _vp, _i, _i, _i, _i, _i, _d, _d, _i, _i, _vp, _i, _i64,
                                      _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "oc_fused_attention_v2_noalloc": (_i, [_vp, _i, _i64, _vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i, _i64, _i,
                                           _d, _i, _i, _vp, _i, _i64, _vp, _vp, _vp, _vp]),
    "oc_tile_high_norms": (_i, [_vp, _i, _i, _i64, _i, _i64, _i64, _i, _i, _vp, _i64, _vp]),
    "oc_decode_gate": (_i, [_vp, _i, _i64, _i, _i, _i, _vp, _i64, _i, _i, _d, _i, _i, _i, _vp, _vp, _vp]),
    "oc_cached_workspace_bytes": (_sz, [_i64, _i, _i64, _i]),
    "oc_fused_attention_cached": (_i, [_vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64,
                                       _i, _i, _i, _i64, _i, _vp, _i64, _i64, _d, _i, _i, _i, _vp, _i, _i64, _i64,
                                       _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "oc_fused_attention_tiles": (_i, [_vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64,
                                      _i, _i, _i, _i64, _i, _vp, _i64, _vp, _i, _vp, _i, _i64, _i64, _vp, _vp, _vp,
                                      _vp, _vp, _vp, _sz, _vp]),
    "oc_lse_merge": (_i, [_vp, _vp, _vp, _i64, _i, _i, _vp, _i, _vp]),
    "oc_add_rms_norm": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, C.c_float, _i, _vp]),
    "oc_rope_cache_append": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i, _vp]),
    "oc_gemv": (_i, [_vp, _vp, _vp, C.c_float, _vp, _vp, _i64, _i64, _i64, _vp, _i, _i, _vp]),
    "oc_gemv_qkv_rope": (_i, [_vp, _vp, _vp, C.c_float, _vp, _vp, _i64, _i64, _i, _i, _i, _vp, _vp, _vp, _vp, _vp,
                              _vp, _i64, _i, _vp]),
    "oc_tail_merge": (_i, [_vp, _i, _i, _i, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, C.c_float, _vp, _i, _vp]),
    "oc_fused_attention_v3_shard": (_i, [_vp, _i, _i64, _vp, _i, _i64, _i64, _vp, _i, _i64, _i64, _i, _i, _i64,
                                         _i, _d, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
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


_binding = None
_binding_tried = False


def binding():
    """The compiled binding (_lib/oc_torch.so) of the hot calls, or None.

    It calls the same C ABI with less host overhead per call than ctypes.
    Not used when ORTHOCACHE_B200_LIB selects another build of the library
    (the binding links the in-tree one).
    """
    global _binding, _binding_tried
    if not _binding_tried:
        _binding_tried = True
        path = os.path.join(_PKG, "_lib", "oc_torch.so")
        if not os.environ.get("ORTHOCACHE_B200_LIB") and os.path.exists(path):
            import importlib.util
            load()
            spec = importlib.util.spec_from_file_location("oc_torch", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            _binding = mod
    return _binding


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


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """Handle of the current CUDA stream of ``device`` (a cudaStream_t as int)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


_sm_cache: dict = {}


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_cache.get(idx)
    if n is None:
        n = _sm_cache[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return n


_splits_cache: dict = {}


def auto_num_splits(num_tiles: int, device: torch.device) -> int:
    """The reference's split heuristic min(SMs, max(1, T/4), T) (fused_eviction.py:556-570)."""
    key = (num_tiles, device.index)
    s = _splits_cache.get(key)
    if s is None:
        s = _splits_cache[key] = load().oc_auto_num_splits(num_tiles, num_sms(device))
    return s


_wsbytes_cache: dict = {}


def workspace_bytes(num_groups: int, group: int, num_tiles: int, head_dim: int) -> int:
    """oc_workspace_bytes; the size depends only on the query group and head_dim."""
    key = (group, head_dim)
    b = _wsbytes_cache.get(key)
    if b is None:
        b = _wsbytes_cache[key] = load().oc_workspace_bytes(max(1, num_groups), group, num_tiles, head_dim)
    return b


class _Workspace:
    """Split-K workspace and control words for one (device, stream).

    The workspace needs no initialisation (every launch writes what it
    reads).  ``ctrl[0]`` receives the retained-tile count of a call (written
    by the launch), ``ctrl[1]`` is the sticky status word: launches OR error
    bits into it and only :func:`read_stats` / :func:`check_status` clear it.
    """

    def __init__(self, device):
        self.device = device
        self.buf = torch.empty(0, dtype=torch.uint8, device=device)
        self.buf_ptr, self.buf_bytes = self.buf.data_ptr(), 0
        self.ctrl = torch.zeros(2, dtype=torch.int32, device=device)
        self.retained_ptr = self.ctrl.data_ptr()
        self.status_ptr = self.retained_ptr + 4
        self.status = self.ctrl[1]  # device view of the status word (handed out in metadata)

    def get(self, nbytes: int):
        """(pointer, size) of a workspace of at least ``nbytes``."""
        if self.buf_bytes < nbytes:
            self.buf = torch.empty(max(nbytes, 2 * self.buf_bytes), dtype=torch.uint8, device=self.device)
            self.buf_ptr, self.buf_bytes = self.buf.data_ptr(), self.buf.numel()
        return self.buf_ptr, self.buf_bytes


_ws: dict = {}


def workspace(device: torch.device, stream: int | None = None) -> _Workspace:
    """The workspace of ``device`` for ``stream`` (default: its current stream)."""
    if stream is None:
        stream = stream_ptr(device)
    key = (device.index, stream)
    w = _ws.get(key)
    if w is None:
        w = _ws[key] = _Workspace(device)
    return w


def _raise_status(status: int) -> None:
    bits = [m for b, m in STATUS_BITS.items() if status & b]
    raise RuntimeError("orthocache_gpu_b200 kernel reported (a launch on this stream since the status was "
                       "last checked): " + "; ".join(bits))


def read_stats(ws: _Workspace) -> int:
    """Synchronising read of the retained-tile count; raises (and clears) a device status."""
    retained, status = ws.ctrl.tolist()
    if status:
        ws.ctrl[1].zero_()
        _raise_status(status)
    return int(retained)


def check_status(device=None) -> None:
    """Raise if a launch on ``device``'s current stream reported an error since the last check.

    Calls made with ``stats=False`` do not synchronise and so cannot raise
    themselves; their errors stay in the stream's sticky status word until
    this function (or the next ``stats=True`` call on the stream) reads it.
    Synchronises with the stream.  Clears the word after reading it.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    ws = workspace(dev)
    status = int(ws.ctrl[1].item())
    if status:
        ws.ctrl[1].zero_()
        _raise_status(status)


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def prepare_kv(t: torch.Tensor) -> torch.Tensor:
    """A view whose last dim is contiguous and whose other strides and base are 16-byte aligned.

    Copies only when the given layout cannot be streamed directly.
    """
    es = t.element_size()
    if t.is_contiguous() and (t.shape[-1] * es) % 16 == 0 and t.data_ptr() % 16 == 0:
        return t  # the common case, checked without walking the strides in Python
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
