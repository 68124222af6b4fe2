"""ctypes binding of libhokv.so (the C ABI in include/hokv.h).

The package has no CPU path: every computation goes through this library on a
CUDA device.  Importing the package works without a GPU (so configuration and
pure bookkeeping stay usable), but the first call that needs the device raises
``RuntimeError`` when CUDA or the library is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

try:
    import torch
    _HAS_TORCH = True
except ImportError:  # pragma: no cover - torch is a hard dependency of the device path
    torch = None
    _HAS_TORCH = False

# HOKV_LIB_VARIANT=stamps loads the profiling build (phase stamps in the decode
# kernels, hokv_phase_stamps); the default is the product library.
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib",
                        "libhokv_stamps.so" if os.environ.get("HOKV_LIB_VARIANT") == "stamps" else "libhokv.so")

F32, F16, BF16, U8, I32, F64 = 0, 1, 2, 3, 4, 5
DOT_SEQ_FMA, DOT_GEMV, DOT_L16_PAIR = 0, 1, 2

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_DEVICE_INPUT, ERR_WORKSPACE = range(7)

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_f32 = ctypes.c_float
_c_f64 = ctypes.c_double
_c_sz = ctypes.c_size_t
_vp = ctypes.c_void_p


class HokvError(RuntimeError):
    """A libhokv entry point returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Cdc03Args(ctypes.Structure):
    """Mirror of ``hokv_cdc03_args`` (include/hokv.h)."""

    _fields_ = [
        ("batch", _c_int), ("kv_heads", _c_int), ("q_per_kv", _c_int), ("head_dim", _c_int),
        ("n_subspaces", _c_int), ("sub_dim", _c_int), ("code_bytes", _c_int), ("cb_slots", _c_int), ("top_k", _c_int),
        ("sink_tokens", _c_int), ("hot_window", _c_int), ("scale", _c_f32), ("lut_order", _c_int),
        ("q", _vp), ("q_dtype", _c_int), ("q_stride_b", _c_i64),
        ("out", _vp), ("out_dtype", _c_int), ("out_stride_b", _c_i64),
        ("k", _vp), ("v", _vp), ("kv_dtype", _c_int), ("kv_stride_b", _c_i64), ("kv_stride_h", _c_i64),
        ("capacity", _c_i64),
        ("codes", _vp), ("code_stride_b", _c_i64), ("code_stride_h", _c_i64),
        ("codebook", _vp), ("cb_stride_b", _c_i64), ("cb_stride_h", _c_i64),
        ("cb_k", _vp), ("cbk_stride_b", _c_i64), ("cbk_stride_h", _c_i64),
        ("seq_len", _vp),
        ("sel_idx", _vp), ("sel_score", _vp), ("sel_count", _vp),
        ("workspace", _vp), ("workspace_bytes", _c_sz),
    ]


_SIGS = {
    "hokv_abi_version": (_c_int, []),
    "hokv_status_string": (ctypes.c_char_p, [_c_int]),
    "hokv_last_error": (ctypes.c_char_p, []),
    "hokv_dot_order_for": (_c_int, [_c_i64, _c_int]),
    "hokv_device_status": (_c_int, [_vp]),
    "hokv_scalar_assign": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp, _c_i64, _c_int, _vp]),
    "hokv_scalar_decode": (_c_int, [_vp, _c_i64, _vp, _c_int, _vp, _vp]),
    "hokv_scalar_kmeans_workspace_size": (_c_sz, [_c_i64, _c_int]),
    "hokv_scalar_kmeans": (_c_int, [_vp, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_f64, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _c_sz, _vp]),
    "hokv_scalar_ema": (_c_int, [_vp, _c_i64, _vp, _c_int, _c_f32, _vp, _c_sz, _vp]),
    "hokv_scalar_ema_workspace_size": (_c_sz, [_c_i64]),
    "hokv_recon_stats": (_c_int, [_vp, _vp, _c_i64, _vp, _vp, _c_sz, _vp]),
    "hokv_scalar_vq_qkt": (_c_int, [_vp, _vp, _c_int, _c_i64, _c_int, _c_i64, _vp, _c_int, _c_f32, _c_int, _vp, _vp]),
    "hokv_pq_assign": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp, _c_int, _c_i64, _vp,
                                _c_i64, _vp, _c_i64, _c_i64, _c_int, _c_int, _vp]),
    "hokv_pq_decode": (_c_int, [_vp, _c_i64, _c_i64, _c_int, _c_int, _vp, _c_int, _vp, _vp]),
    "hokv_vq_kmeans_workspace_size": (_c_sz, [_c_i64, _c_int, _c_int]),
    "hokv_vq_kmeans": (_c_int, [_vp, _c_i64, _c_int, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_f64, _vp, _c_int,
                                _vp, _vp, _vp, _vp, _c_sz, _vp]),
    "hokv_pq_tables": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_i64, _vp, _c_i64, _vp, _vp, _c_int,
                                _vp]),
    "hokv_pq_gather": (_c_int, [_vp, _c_int, _c_int, _vp, _c_i64, _c_i64, _c_int, _c_f32, _vp, _vp]),
    "hokv_pq_value_output": (_c_int, [_vp, _c_i64, _vp, _c_i64, _c_int, _c_int, _vp, _c_int, _vp, _vp, _vp, _c_sz,
                                      _vp]),
    "hokv_pq_value_output_workspace_size": (_c_sz, [_c_int]),
    "hokv_cdc03_workspace_size": (_c_int, [ctypes.POINTER(Cdc03Args), ctypes.POINTER(_c_sz)]),
    "hokv_cdc03_decode": (_c_int, [ctypes.POINTER(Cdc03Args), _vp]),
    "hokv_cdc03_candidates": (_c_int, [ctypes.POINTER(Cdc03Args), _vp]),
    "hokv_cdc03_attend": (_c_int, [ctypes.POINTER(Cdc03Args), _vp]),
    "hokv_cdc03_decode_noalloc": (_c_int, [ctypes.POINTER(Cdc03Args), _vp]),
    "hokv_age_tokens": (_c_int, [ctypes.POINTER(Cdc03Args), _vp, _vp, _c_int, _vp]),
    "hokv_dense_attention": (_c_int, [_vp, _vp, _vp, _c_int, _c_i64, _c_int, _c_f64, _c_int, _vp, _vp, _vp, _vp,
                                      _c_sz, _vp]),
    "hokv_prefill_attention": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int]
                               + [_c_i64] * 12 + [_c_f32, _c_int, _vp]),
    "hokv_softmax": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _c_sz, _vp]),
    "hokv_prefilter_mask": (_c_int, [_vp, _c_int, _vp, _c_i64, _c_int, _vp, _vp]),
    "hokv_scale_f32_to_f64": (_c_int, [_vp, _c_i64, _c_f64, _vp, _vp]),
    "hokv_phase_stamps": (_c_int, [_vp, _c_sz]),
}

_lock = threading.Lock()
_lib = None


def lib():
    """Load libhokv.so once; raise if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libhokv.so not found at {LIB_PATH}: build it first "
                        "(python -c 'import __graft_entry__ as g; g.build()')")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def available() -> bool:
    """True when the CUDA device path can run (the old ``_HAS_TRITON`` meaning)."""
    if not _HAS_TORCH or not torch.cuda.is_available():
        return False
    try:
        lib()
    except (RuntimeError, OSError):
        return False
    return True


def require_device():
    """Raise unless a CUDA device and the library are present (no CPU fallback)."""
    if not _HAS_TORCH:
        raise RuntimeError("helix_online_kv needs torch with CUDA; it has no CPU path")
    if not torch.cuda.is_available():
        raise RuntimeError("helix_online_kv runs on a CUDA device (B200); no CUDA device is visible "
                           "and there is no CPU fallback")
    lib()


def check(status: int, what: str = ""):
    if status != OK:
        msg = lib().hokv_last_error().decode(errors="replace")
        raise HokvError(status, f"{what}: {msg}" if what else msg)


def stream():
    return _vp(torch.cuda.current_stream().cuda_stream)


def ptr(t):
    return _vp(t.data_ptr()) if t is not None else _vp(0)


def device():
    return torch.device("cuda", torch.cuda.current_device())


def dtype_code(t) -> int:
    return {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.uint8: U8,
            torch.int32: I32, torch.float64: F64}[t.dtype]


def to_dev(a, dtype=None):
    """numpy / torch input -> contiguous CUDA tensor (float32 unless dtype given)."""
    if isinstance(a, torch.Tensor):
        t = a.detach()
        if dtype is not None:
            t = t.to(dtype)
        return t.to(device()).contiguous()
    arr = np.asarray(a)
    if dtype is None:
        dtype = torch.float32
    np_dt = {torch.float32: np.float32, torch.float64: np.float64, torch.uint8: np.uint8,
             torch.int32: np.int32, torch.float16: np.float16}[dtype]
    arr = np.ascontiguousarray(arr, dtype=np_dt)
    return torch.from_numpy(arr).to(device(), non_blocking=False)


def workspace(nbytes: int):
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device())


def device_status():
    check(lib().hokv_device_status(stream()), "device")


def dot_order_for(n_rows: int, dim: int) -> int:
    if n_rows == 1:
        return DOT_GEMV
    if n_rows <= 4 and dim >= 32:
        return DOT_L16_PAIR
    return DOT_SEQ_FMA
