"""ctypes binding of libmaba_b200.so (the C ABI declared in include/maba_b200.h).

Torch tensors cross the boundary as ``maba_tensor`` descriptors (device
pointer, dtype code, shape, element strides); streams as raw ``cudaStream_t``
values.  There is no CPU implementation behind this module: when the library
is missing, or a tensor is not on a CUDA device, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmaba_b200.so"

MAX_DIMS = 6
DTYPE_CODES = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.float64: 3,
    torch.int64: 4,
    torch.int32: 5,
}

# status codes of include/maba_b200.h
OK, ERR_INVALID, ERR_DTYPE, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = range(6)


class MabaTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


T_P = ctypes.POINTER(MabaTensor)
_i32, _i64, _f32, _vp, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes); the exact set of entry points of include/maba_b200.h
SIGNATURES = {
    "maba_abi_version": (ctypes.c_int, []),
    "maba_last_error": (ctypes.c_char_p, []),
    "maba_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32), _vp]),
    "maba_selftest_wait_timeout": (ctypes.c_int, [_i64, _vp]),
    "maba_dgda_prefill": (ctypes.c_int, [T_P] * 10 + [_i32, _vp, _sz, _vp]),
    "maba_dgda_prefill_workspace_size": (_sz, [_i32, _i64, _i64, _i64, _i64, _i64]),
    "maba_dgda_step": (ctypes.c_int, [T_P] * 10 + [_vp]),
    "maba_dgda_transition": (ctypes.c_int, [T_P] * 8 + [_vp, _sz, _vp]),
    "maba_dgda_frontend": (ctypes.c_int, [T_P] * 5 + [_i32, _f32, _vp]),
    "maba_rmsnorm_residual": (ctypes.c_int, [T_P, T_P, T_P, T_P, _f32, T_P, _vp]),
    "maba_swiglu": (ctypes.c_int, [T_P, T_P, _vp]),
    "maba_decode_gemv": (ctypes.c_int, [T_P, _i32, T_P, T_P, _f32, T_P, _i32, T_P, T_P, T_P, T_P, T_P, _i32, _i32,
                                        T_P, _vp, _vp, _sz, _vp]),
    "maba_decode_gemv_workspace_size": (_sz, [_i64]),
    "maba_decode_dgda_state": (ctypes.c_int, [T_P, T_P, T_P, _i32, _f32, _vp]),
    "maba_decode_dgda_mix": (ctypes.c_int, [T_P, T_P, T_P, _f32, T_P, T_P, T_P, T_P, T_P, _i32, _f32, _vp, _sz, _vp]),
    "maba_decode_dgda_mix_workspace_size": (ctypes.c_size_t, [_i32]),
    "maba_dgda_transition_workspace_size": (_sz, [_i32, _i64, _i64, _i64]),
    "maba_compute_centroids": (ctypes.c_int, [T_P, T_P, _i32, _vp]),
    "maba_index_topk": (ctypes.c_int, [T_P, T_P, _f32, _i32, _i32, _i32, T_P, T_P, _vp, _sz, _vp]),
    "maba_index_topk_workspace_size": (_sz, [_i64, _i64, _i64, _i32]),
    "maba_index_topk_at": (ctypes.c_int, [T_P, T_P, _f32, _i32, _i32, _i64, T_P, T_P, _vp, _sz, _vp]),
    "maba_index_topk_at_workspace_size": (_sz, [_i64, _i64, _i64, _i32, _i32, _i64]),
    "maba_index_topk_noalloc": (ctypes.c_int, [T_P, T_P, _f32, _i32, _i32, _i32, T_P, T_P, _vp]),
    "maba_stream_superposition": (ctypes.c_int, [T_P, T_P, T_P, T_P, _i32, T_P, _vp]),
    "maba_hca_pool": (ctypes.c_int, [T_P, T_P, _i32, _vp]),
    "maba_sa_attention": (ctypes.c_int, [T_P] * 6 + [_i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "maba_sa_attention_workspace_size": (_sz, [_i32, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32]),
    "maba_decode_cache_append": (ctypes.c_int, [T_P] * 6 + [_vp, _i32, _i32, _vp]),
    "maba_index_topk_decode_at": (ctypes.c_int, [T_P, T_P, _f32, _i32, _i32, _vp, T_P, _vp, _sz, _vp]),
    "maba_index_topk_decode_at_workspace_size": (_sz, [_i64, _i64, _i32]),
    "maba_sa_attention_decode_at": (ctypes.c_int, [T_P] * 6 + [_vp, _i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "maba_sa_attention_decode_at_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32]),
}

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def load_library(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Load (once) and return the native library, with typed entry points."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"maba_b200 native library not found at {p}; build it with "
                "`python -m maba_v2_architecture_b200.build` (there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.maba_abi_version() != 1:
            raise RuntimeError("maba_b200: ABI version mismatch between Python and libmaba_b200.so")
        if path is None:
            _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return load_library()


def desc(t: Optional[torch.Tensor]) -> Optional[MabaTensor]:
    """Descriptor of a device tensor (None for an absent operand)."""
    if t is None:
        return None
    if t.dim() > MAX_DIMS:
        raise ValueError(f"maba_b200: tensors up to {MAX_DIMS} dims, got {t.dim()}")
    code = DTYPE_CODES.get(t.dtype)
    if code is None:
        raise TypeError(f"maba_b200: unsupported dtype {t.dtype}")
    d = MabaTensor()
    d.data = t.data_ptr() if t.numel() > 0 else None
    d.dtype = code
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.shape[i] = s
        d.stride[i] = st
    return d


def ref(d: Optional[MabaTensor]):
    return ctypes.byref(d) if d is not None else None


def desc_array(tensors) -> ctypes.Array:
    """Contiguous array of descriptors (an absent operand has NULL data), for the entry
    points that take a fixed-length list of tensors."""
    arr = (MabaTensor * len(tensors))()
    for i, t in enumerate(tensors):
        if t is not None:
            arr[i] = desc(t)
    return arr


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    msg = lib().maba_last_error().decode(errors="replace")
    if rc == ERR_INVALID:
        raise ValueError(msg)
    if rc == ERR_DTYPE:
        raise TypeError(msg)
    raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def require_cuda(*tensors: Optional[torch.Tensor], op: str) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError(
                f"maba_b200.{op}: tensors must be on a CUDA device (got {t.device}); "
                "this backend has no CPU path"
            )


_ws_cache: dict = {}
_ws_lock = threading.Lock()


def workspace(nbytes: int, device: torch.device) -> Optional[torch.Tensor]:
    """Scratch for one op call, reused across calls on the same device and stream.

    Ops on one stream run in order, so consecutive calls can share the buffer; a
    larger request replaces it.  Keeping it avoids a several-hundred-MB allocation
    per call (the DGDA record buffer), which the caching allocator could turn into a
    blocking cudaMalloc in the middle of a stream of launches."""
    if nbytes <= 0:
        return None
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    with _ws_lock:
        bufs = _ws_cache.setdefault(key, [])
        if not bufs or bufs[-1].numel() < nbytes:
            # smaller buffers stay alive: a captured CUDA graph may still point at them
            bufs.append(torch.empty(int(nbytes), dtype=torch.uint8, device=dev))
        return bufs[-1]


def release_workspaces() -> None:
    """Drops the cached per-stream scratch buffers (they are re-created on demand); only
    safe when no captured CUDA graph still uses them."""
    with _ws_lock:
        _ws_cache.clear()


def device_error(device: Optional[torch.device] = None) -> int:
    """Reads and clears the device error word of the current device (0 = no kernel gave up on a wait)."""
    out = ctypes.c_int32(0)
    stream = torch.cuda.current_stream(device).cuda_stream
    check(lib().maba_device_error(ctypes.byref(out), ctypes.c_void_p(stream)), "maba_device_error")
    return int(out.value)
