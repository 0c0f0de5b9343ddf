"""ctypes binding of libinferd_sm100a.so (the C ABI declared in include/inferd_b200.h).

There is no CPU path: every function here needs CUDA tensors and the built library, and
raises RuntimeError when either is missing.  Status codes map to the exception types
the reference raises for the same conditions (ValueError for argument errors,
IndexError for block ids outside the pool).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libinferd_sm100a.so"

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE_INDEX = 5
ERR_DEVICE_TIMEOUT = 6

DTYPE_CODES = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.float8_e4m3fn: 3,
}

_lib = None
_lock = threading.Lock()

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/inferd_b200.h
_SIGNATURES = {
    "inferd_version": (ctypes.c_int, []),
    "inferd_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "inferd_last_cuda_error": (ctypes.c_char_p, []),
    "inferd_host_device_pointer": (ctypes.c_int, [_c_void_p, _c_void_p]),
    "inferd_reshape_and_cache": (ctypes.c_int, [
        _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64,
        _i32, _i32, _i32, _i64, _i32, _c_void_p, _c_void_p]),
    "inferd_gather_paged_kv": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64, _i32, _i32, _i32,
        _i64, _i32, _c_void_p, _c_void_p]),
    "inferd_paged_attention": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64, _c_void_p, _i32,
        _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _i32, _c_void_p, _sz, _c_void_p,
        _c_void_p]),
    "inferd_paged_attention_noalloc": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64, _c_void_p, _i32,
        _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _i32, _c_void_p, _c_void_p]),
    "inferd_paged_attention_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "inferd_paged_attention_counter_bytes": (_sz, [_i32, _i32]),
    "inferd_dense_attention": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32, _f32, _i32,
        _c_void_p]),
    "inferd_fp8_quantize_per_channel": (ctypes.c_int, [
        _c_void_p, _i32, _c_void_p, _c_void_p, _i64, _i64, _c_void_p]),
    "inferd_fp8_linear": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p, _sz,
        _c_void_p]),
    "inferd_fp8_packed_weight_bytes": (_sz, [_i64, _i64]),
    "inferd_fp8_pack_weights": (ctypes.c_int, [_c_void_p, _c_void_p, _i64, _i64, _c_void_p]),
    "inferd_fp8_linear_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32]),
    "inferd_block_tables_refresh": (ctypes.c_int, [
        _c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p]),
    "inferd_fp8_quantize_dynamic": (ctypes.c_int, [
        _c_void_p, _i32, _c_void_p, _c_void_p, _i64, _i64, _i32, _c_void_p, _c_void_p]),
    "inferd_fp8_dynamic_linear": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _i32, _c_void_p, _sz,
        _c_void_p]),
    "inferd_nucleus_sample": (ctypes.c_int, [
        _c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i64, _i32, _i64, _c_void_p, _f32,
        _c_void_p, _f32, _u64, _u64, _c_void_p, _c_void_p]),
    "inferd_sample_probs": (ctypes.c_int, [
        _c_void_p, _c_void_p, _i64, _i32, _i64, _u64, _u64, _c_void_p, _c_void_p]),
    "inferd_spec_accept": (ctypes.c_int, [
        _c_void_p, _c_void_p, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64,
        _i32, _i32, _i64, _u64, _u64, _c_void_p, _c_void_p]),
    "inferd_peer_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(_c_void_p), _c_void_p]),
    "inferd_peer_open": (ctypes.c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "inferd_peer_close": (ctypes.c_int, [_c_void_p]),
    "inferd_peer_free": (ctypes.c_int, [_c_void_p]),
    "inferd_gather_push": (ctypes.c_int, [
        _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, ctypes.c_uint32, _c_void_p]),
    "inferd_paged_attention_gather": (ctypes.c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64, _c_void_p, _i32,
        _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _i32, _c_void_p, _sz, _c_void_p, _i32,
        _i64, _c_void_p, _c_void_p]),
    "inferd_gather_publish": (ctypes.c_int, [_c_void_p, _i32, _i32, ctypes.c_uint32, _c_void_p]),
    "inferd_paged_attention_reserve_sms": (ctypes.c_int, [_i32]),
    "inferd_paged_attention_reserved_sms": (_i32, []),
    "inferd_gather_wait": (ctypes.c_int, [
        _c_void_p, _i32, ctypes.c_uint32, _u64, _c_void_p, _c_void_p]),
}

IPC_HANDLE_BYTES = 64


def exported_symbols() -> list[str]:
    """Names the binding expects the library to export (every entry point of the header)."""
    return list(_SIGNATURES)


def load(path: Path | str | None = None):
    """Load (once) and return the ctypes handle of libinferd_sm100a.so."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is not built; run `python -m inferd_b200.build` "
                "(inferd_b200 has no CPU fallback)")
        handle = ctypes.CDLL(str(p))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = handle
        return handle


def status_message(status: int) -> str:
    lib = load()
    msg = lib.inferd_status_string(status).decode()
    if status == ERR_CUDA:
        cuda = lib.inferd_last_cuda_error().decode()
        if cuda:
            msg = f"{msg}: {cuda}"
    return msg


def check(status: int, what: str) -> None:
    """Raise the exception the reference would raise for this status."""
    if status == OK:
        return
    msg = f"{what}: {status_message(status)}"
    if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED):
        raise ValueError(msg)
    if status == ERR_DEVICE_INDEX:
        raise IndexError(msg)
    raise RuntimeError(msg)


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors must live on one CUDA device; there is no CPU implementation."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(
                f"inferd_b200 kernels run on CUDA tensors only (got a tensor on {t.device}); "
                "there is no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def check_out(out: torch.Tensor, device: torch.device, what: str) -> None:
    """An output tensor the kernels write through its raw pointer must be on the inputs'
    CUDA device: a host tensor (pinned or not) or another GPU's would hand the kernel an
    address it must not write."""
    if out.device != device:
        raise ValueError(f"{what}: out is on {out.device}, the inputs on {device}")


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


# ---------------------------------------------------------------- per-device state
class _DeviceState:
    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.error_word = torch.zeros(1, dtype=torch.int32, device=device)
        self.workspace: torch.Tensor | None = None


_states: dict[int, _DeviceState] = {}


def device_state(device: torch.device) -> _DeviceState:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _states.get(idx)
    if st is None:
        st = _DeviceState(torch.device("cuda", idx))
        _states[idx] = st
    return st


def error_word(device: torch.device) -> torch.Tensor:
    return device_state(device).error_word


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Shared attention workspace of at least nbytes, zero-initialised on (re)allocation.

    The kernels leave the ticket counters at its head zero after every completed call, so
    one workspace serves every call ordered on the same stream.
    """
    st = device_state(device)
    if st.workspace is None or st.workspace.numel() < nbytes:
        st.workspace = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=st.device)
    return st.workspace


def raise_device_errors(device: torch.device) -> None:
    """Synchronise on the device's error word; raise and clear it if a kernel set it."""
    st = device_state(device)
    code = int(st.error_word.item())
    if code != OK:
        st.error_word.zero_()
        check(code, "device-side check")
