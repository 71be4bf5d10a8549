"""ctypes binding of libmicroinfer_b200.so (the C ABI in include/microinfer_b200.h).

The library is loaded once per process.  There is no fallback: if the shared
object is missing, or a call is made with CPU tensors, the wrappers raise.
Status codes follow the C ABI: negative -> ``ValueError`` (argument rejected,
nothing launched), positive -> ``RuntimeError`` (CUDA launch error).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmicroinfer_b200.so"

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
INDEX_CODES = {torch.int32: 0, torch.int64: 1}

DEV_BAD_BLOCK = 1
DEV_BAD_SLOT = 2
DEV_TIMEOUT = 4
DEV_BAD_POSITION = 8
DEV_BAD_ROW = 16

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/microinfer_b200.h
SIGNATURES = {
    "mi_abi_version": (ctypes.c_int, []),
    "mi_last_error": (ctypes.c_char_p, []),
    "mi_device_sm_count": (ctypes.c_int, [ctypes.c_int]),
    "mi_store_kv": (
        ctypes.c_int,
        [_P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _I32, _P, _P, _I64, _I64, _I64, _P, _P],
    ),
    "mi_store_kv_slots": (
        ctypes.c_int,
        [_P, _P, _I64, _I32, _I32, _I32, _I32, _P, _I32, _P, _P, _I64, _I64, _I64, _P, _P],
    ),
    "mi_paged_decode_workspace_bytes": (_SZ, [_I64, _I32, _I32, _I32]),
    "mi_paged_decode_default_splits": (ctypes.c_int, [_I64, _I32, _I32, ctypes.c_int]),
    "mi_paged_decode": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _F, _I32, _P,
         _SZ, _P, _P],
    ),
    "mi_paged_decode_uses_workspace": (ctypes.c_int, [_I32]),
    "mi_paged_decode_plan": (
        ctypes.c_int,
        [_I64, _I32, _I32, _I32, _I32, _I32, _I64, _I32, ctypes.c_int, ctypes.POINTER(_I32),
         ctypes.POINTER(_SZ)],
    ),
    "mi_paged_decode_store": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _P, _P, _I64, _P,
         _F, _I32, _I32, _P, _SZ, _P, _P],
    ),
    "mi_paged_decode_noalloc": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _F, _I32, _P,
         _P],
    ),
    "mi_prefill_kernel_for": (ctypes.c_int, [_I32, _I32, _I32, _I32, _I32]),
    "mi_paged_prefill": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _I64, _I64, _I64, _I32,
         _F, _P, _P],
    ),
    "mi_varlen_prefill": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _I64, _I64, _I64, _I32, _F, _P,
         _P],
    ),
    "mi_gather_paged_kv": (
        ctypes.c_int,
        [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _I64, _I32, _P, _P],
    ),
    "mi_copy_blocks": (ctypes.c_int, [_P, _P, _I32, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "mi_wait_flag_selftest": (ctypes.c_int, [_P, _I64, _P, _P]),
    "mi_build_decode_metadata": (
        ctypes.c_int,
        [_P, _I32, _I32, _P, _I32, _P, _I32, _I32, _I64, _I32, _P, _P, _P, _P, _P, _P, _P],
    ),
    "mi_build_prefill_metadata": (
        ctypes.c_int,
        [_P, _I32, _I32, _P, _I32, _P, _I32, _P, _I64, _I32, _I64, _I32, _P, _P, _P, _P, _P, _P,
         _P, _P],
    ),
    "mi_qk_norm_rope_store": (
        ctypes.c_int,
        [_P, _I64, _P, _I64, _P, _P, _F, _P, _I32, _P, _P, _I64, _I32, _P, _P, _P, _I64, _I32,
         _I64, _I32, _I32, _I32, _I32, _P, _P],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the shared library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m microinfer_b200.build` "
                    "(or __graft_entry__.build())"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int) -> None:
    if status == 0:
        return
    msg = load().mi_last_error().decode(errors="replace")
    if status < 0:
        raise ValueError(msg)
    raise RuntimeError(f"CUDA error {status}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def index_code(dtype: torch.dtype) -> int:
    try:
        return INDEX_CODES[dtype]
    except KeyError:
        raise ValueError(f"index tensors must be int32 or int64, got {dtype}") from None


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    """All given tensors must live on one CUDA device; returns it."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(
                "microinfer_b200 kernels need CUDA tensors (there is no CPU path); "
                f"got a tensor on {t.device}"
            )
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"tensors on different devices: {device} and {t.device}")
    if device is None:
        raise ValueError("no tensor given")
    return device


_status_buffers: dict[int, torch.Tensor] = {}


def status_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR MI_DEV_* bits into."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status_buffers.get(index)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _status_buffers[index] = buf
    return buf


def read_device_status(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Synchronise and return (optionally clearing) the device status word."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    buf = status_buffer(device)
    value = int(buf.item())
    if reset and value:
        buf.zero_()
    return value


def check_device_status(device: torch.device | int | None = None) -> None:
    """Raise if any kernel on `device` reported a bad id or a timeout."""
    value = read_device_status(device)
    if value:
        reasons = []
        if value & DEV_BAD_BLOCK:
            reasons.append("block id outside the pool")
        if value & DEV_BAD_SLOT:
            reasons.append("slot outside the cache")
        if value & DEV_TIMEOUT:
            reasons.append("bounded wait timed out")
        raise RuntimeError("device status: " + ", ".join(reasons))
