"""ctypes binding of the C ABI in ``include/kata_b200.h`` (``libkata_b200.so``).

This module is the only place that touches the shared library.  It mirrors the argument
structs field for field, converts torch tensors to raw device pointers and sizes, and turns
nonzero return codes into ``RuntimeError`` with the library's own message.  There is no CPU
or framework fallback: if the library is missing, or a tensor is not on a CUDA device, every
call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "libkata_b200.so"

KATA_OK = 0
DTYPE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
ALGO = {"auto": 0, "tc": 1, "simt": 2, "tc_gram": 3}
SCORE = {"concat": 0, "sum": 1}
ABI_VERSION = 2

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("g", c_void_p), ("state", c_void_p),
        ("o", c_void_p), ("den", c_void_p), ("work", c_void_p),
        ("dtype", c_int), ("B", c_int), ("HQ", c_int), ("H", c_int), ("D", c_int), ("Dv", c_int),
        ("M", c_int), ("lds", c_int), ("score", c_int), ("scale", c_float),
    ]


class AttnFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("c", c_void_p),
        ("o", c_void_p), ("den", c_void_p), ("status", c_void_p),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("H", c_int), ("HQ", c_int), ("D", c_int), ("Dv", c_int),
        ("M", c_int), ("score", c_int), ("algo", c_int), ("scale", c_float),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("cu_seqlens", c_void_p), ("num_seqs", c_int),
    ]


class AttnBwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("o", c_void_p), ("den", c_void_p),
        ("dout", c_void_p), ("c", c_void_p), ("dq", c_void_p), ("dk", c_void_p), ("dv", c_void_p),
        ("dc", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("status", c_void_p),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("H", c_int), ("HQ", c_int), ("D", c_int), ("Dv", c_int),
        ("M", c_int), ("score", c_int), ("algo", c_int), ("scale", c_float), ("phases", c_int),
        ("cu_seqlens", c_void_p), ("num_seqs", c_int),
    ]


class DeltaFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("beta", c_void_p),
        ("U", c_void_p), ("E", c_void_p), ("o", c_void_p), ("den", c_void_p),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("H", c_int), ("D", c_int), ("Dv", c_int),
        ("M", c_int), ("normalize", c_int), ("scale", c_float), ("eps", c_float), ("phases", c_int),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("state", c_void_p),
    ]


class DeltaBwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("beta", c_void_p),
        ("U", c_void_p), ("E", c_void_p), ("o", c_void_p), ("den", c_void_p), ("dout", c_void_p), ("z", c_void_p),
        ("dq", c_void_p), ("dk", c_void_p), ("dv", c_void_p), ("dbeta", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("H", c_int), ("D", c_int), ("Dv", c_int),
        ("M", c_int), ("normalize", c_int), ("scale", c_float), ("eps", c_float),
    ]


class GdnFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("g", c_void_p), ("beta", c_void_p), ("h0", c_void_p),
        ("o", c_void_p), ("ht", c_void_p), ("A", c_void_p), ("cu_seqlens", c_void_p), ("chunk_offsets", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("H", c_int), ("HV", c_int), ("K", c_int), ("V", c_int),
        ("N", c_int), ("num_chunks", c_int), ("scale", c_float), ("algo", c_int),
    ]


class GdnBwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("g", c_void_p), ("beta", c_void_p), ("h0", c_void_p),
        ("A", c_void_p), ("dout", c_void_p), ("dht", c_void_p), ("dq", c_void_p), ("dk", c_void_p),
        ("dv", c_void_p), ("dg", c_void_p), ("dbeta", c_void_p), ("dh0", c_void_p),
        ("cu_seqlens", c_void_p), ("chunk_offsets", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("fwd_workspace", c_void_p),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("H", c_int), ("HV", c_int), ("K", c_int), ("V", c_int),
        ("N", c_int), ("num_chunks", c_int), ("scale", c_float), ("algo", c_int), ("grad_dtype", c_int),
    ]


class ConvArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("w", c_void_p), ("bias", c_void_p), ("y", c_void_p), ("dy", c_void_p), ("dx", c_void_p),
        ("dw", c_void_p), ("dbias", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("dtype", c_int), ("B", c_int), ("T", c_int), ("C", c_int), ("K", c_int),
        ("ldx", ctypes.c_longlong), ("ldy", ctypes.c_longlong), ("lddx", ctypes.c_longlong), ("activation", c_int),
    ]


class RowNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("w", c_void_p), ("cos", c_void_p), ("sin", c_void_p), ("y", c_void_p), ("rstd", c_void_p),
        ("dy", c_void_p), ("dx", c_void_p), ("dw", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("dtype", c_int), ("rows", ctypes.c_longlong), ("N", c_int), ("T", c_int), ("heads", c_int),
        ("norm", c_int), ("rope", c_int), ("R", c_int), ("eps", c_float),
    ]


class AddRmsNormArgs(ctypes.Structure):
    _fields_ = [
        ("h", c_void_p), ("x", c_void_p), ("w", c_void_p), ("h_out", c_void_p), ("y", c_void_p), ("rstd", c_void_p),
        ("dy", c_void_p), ("dh_in", c_void_p), ("dh", c_void_p), ("dx", c_void_p), ("dw", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("rows", ctypes.c_longlong), ("N", c_int),
        ("dtype", c_int), ("eps", c_float),
    ]


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"{_LIB_PATH.name} is not built; run `python -m linatt_b200.build` "
                    "(nvcc with sm_100a support is required)")
            L = ctypes.CDLL(str(_LIB_PATH))
            L.kata_strerror.restype = ctypes.c_char_p
            L.kata_strerror.argtypes = [c_int]
            L.kata_abi_version.restype = c_int
            L.kata_attn_fwd.restype = c_int
            L.kata_attn_fwd.argtypes = [ctypes.POINTER(AttnFwdArgs), c_void_p]
            L.kata_attn_algo.restype = c_int
            L.kata_attn_algo.argtypes = [ctypes.POINTER(AttnFwdArgs)]
            L.kata_attn_fwd_workspace_bytes.restype = c_size_t
            L.kata_attn_fwd_workspace_bytes.argtypes = [ctypes.POINTER(AttnFwdArgs)]
            L.kata_attn_bwd.restype = c_int
            L.kata_attn_bwd.argtypes = [ctypes.POINTER(AttnBwdArgs), c_void_p]
            L.kata_attn_bwd_noalloc.restype = c_int
            L.kata_attn_bwd_noalloc.argtypes = [ctypes.POINTER(AttnBwdArgs), c_void_p]
            L.kata_attn_bwd_workspace_bytes.restype = c_size_t
            L.kata_attn_bwd_workspace_bytes.argtypes = [ctypes.POINTER(AttnBwdArgs)]
            L.kata_delta_fwd.restype = c_int
            L.kata_delta_fwd.argtypes = [ctypes.POINTER(DeltaFwdArgs), c_void_p]
            L.kata_delta_fwd_workspace_bytes.restype = c_size_t
            L.kata_delta_fwd_workspace_bytes.argtypes = [ctypes.POINTER(DeltaFwdArgs)]
            L.kata_delta_bwd.restype = c_int
            L.kata_delta_bwd.argtypes = [ctypes.POINTER(DeltaBwdArgs), c_void_p]
            L.kata_delta_bwd_workspace_bytes.restype = c_size_t
            L.kata_delta_bwd_workspace_bytes.argtypes = [ctypes.POINTER(DeltaBwdArgs)]
            for nm, st in (("fwd", GdnFwdArgs), ("bwd", GdnBwdArgs)):
                f = getattr(L, f"kata_gdn_{nm}")
                f.restype = c_int
                f.argtypes = [ctypes.POINTER(st), c_void_p]
                w = getattr(L, f"kata_gdn_{nm}_workspace_bytes")
                w.restype = c_size_t
                w.argtypes = [ctypes.POINTER(st)]
            L.kata_sp_features.restype = c_int
            L.kata_sp_features.argtypes = [c_void_p, c_void_p] + [c_int] * 6 + [c_float, c_void_p]
            L.kata_sum_features.restype = c_int
            L.kata_sum_features.argtypes = [c_void_p, c_void_p] + [c_int] * 6 + [c_float, c_void_p]
            L.kata_sp_contract.restype = c_int
            L.kata_sp_contract.argtypes = [c_void_p, c_void_p, c_void_p] + [c_int] * 6 + [c_float, c_int, c_void_p]
            L.kata_sp_combine.restype = c_int
            L.kata_sp_combine.argtypes = [c_void_p] * 5 + [c_int] * 6 + [c_void_p]
            L.kata_sp_bwd_prep.restype = c_int
            L.kata_sp_bwd_prep.argtypes = [c_void_p] * 4 + [c_int] * 6 + [c_void_p]
            L.kata_decode_workspace_bytes.restype = c_size_t
            L.kata_decode_workspace_bytes.argtypes = [ctypes.POINTER(DecodeArgs)]
            L.kata_decode_step.restype = c_int
            L.kata_decode_step.argtypes = [ctypes.POINTER(DecodeArgs), c_void_p]
            L.kata_selftest_umma.restype = c_int
            L.kata_selftest_umma.argtypes = [c_void_p, c_void_p, c_void_p] + [c_int] * 8 + [c_void_p]
            L.kata_sp_state.restype = c_int
            L.kata_sp_state.argtypes = ([c_void_p, c_void_p, c_void_p] + [c_int] * 9 +
                                        [c_float, c_int, c_int, c_void_p, c_void_p])
            L.kata_sp_apply.restype = c_int
            L.kata_sp_apply.argtypes = ([c_void_p, c_void_p, c_void_p] + [c_int] * 8 +
                                        [c_float, c_int, c_int, c_void_p, c_void_p])
            L.kata_sp_grad.restype = c_int
            L.kata_sp_grad.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p] + [c_int] * 7 + [c_float, c_void_p, c_void_p]
            L.kata_selftest_umma_m64.restype = c_int
            L.kata_selftest_umma_m64.argtypes = [c_void_p, c_void_p, c_void_p] + [c_int] * 5 + [c_void_p]
            L.kata_selftest_umma_pair.restype = c_int
            L.kata_selftest_umma_pair.argtypes = [c_void_p, c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]
            for nm, st in (("short_conv", ConvArgs), ("rownorm", RowNormArgs)):
                for ph in ("fwd", "bwd"):
                    f = getattr(L, f"kata_{nm}_{ph}")
                    f.restype = c_int
                    f.argtypes = [ctypes.POINTER(st), c_void_p]
                w = getattr(L, f"kata_{nm}_bwd_workspace_bytes")
                w.restype = c_size_t
                w.argtypes = [ctypes.POINTER(st)]
            c_ll = ctypes.c_longlong
            L.kata_swiglu_fwd.restype = c_int
            L.kata_swiglu_fwd.argtypes = [c_void_p, c_void_p, c_ll, c_int, c_int, c_void_p]
            L.kata_swiglu_bwd.restype = c_int
            L.kata_swiglu_bwd.argtypes = [c_void_p, c_void_p, c_void_p, c_ll, c_int, c_int, c_void_p]
            L.kata_cross_entropy_fwd.restype = c_int
            L.kata_cross_entropy_fwd.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_ll, c_int, c_int, c_void_p]
            L.kata_cross_entropy_bwd.restype = c_int
            L.kata_cross_entropy_bwd.argtypes = [c_void_p] * 6 + [c_ll, c_int, c_int, c_void_p]
            for nm in ("fwd", "bwd"):
                f = getattr(L, f"kata_add_rmsnorm_{nm}")
                f.restype = c_int
                f.argtypes = [ctypes.POINTER(AddRmsNormArgs), c_void_p]
            L.kata_add_rmsnorm_bwd_workspace_bytes.restype = c_size_t
            L.kata_add_rmsnorm_bwd_workspace_bytes.argtypes = [ctypes.POINTER(AddRmsNormArgs)]
            if L.kata_abi_version() != ABI_VERSION:
                raise RuntimeError(f"libkata_b200 ABI {L.kata_abi_version()} != expected {ABI_VERSION}")
            _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != KATA_OK:
        msg = lib().kata_strerror(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (code {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("linatt_b200 kernels run on CUDA tensors only (got a tensor on "
                               f"{t.device}); there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def stream_handle(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


# Per-device status word that bounded device-side waits write on timeout.
_status: dict[int, torch.Tensor] = {}


def status_word(dev: torch.device) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _status[idx] = t
    return t


def check_device_status(dev: torch.device | None = None) -> None:
    """Synchronise and raise if any kernel on ``dev`` reported a bounded-wait timeout."""
    devs = [dev] if dev is not None else [torch.device("cuda", i) for i in _status]
    for d in devs:
        t = status_word(d)
        v = int(t.item())
        if v != 0:
            t.zero_()
            raise RuntimeError(f"linatt_b200 device status {v}: a kernel wait timed out on {d}")


SYNC_CHECK = os.environ.get("KATA_SYNC_CHECK", "0") == "1"
