"""ctypes binding of libmfd_b200.so (include/mfd_b200.h).

The library is the only compute path: if it is missing it is built in-tree with nvcc, and if that fails,
or no CUDA device is present, every call raises.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmfd_b200.so")

_lock = threading.Lock()
_lib = None

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_f32 = ctypes.c_float
c_size = ctypes.c_size_t
c_vp = ctypes.c_void_p

# name -> (restype, argtypes)
_SIGS = {
    "mfd_last_error": (ctypes.c_char_p, []),
    "mfd_abi_version": (c_int, []),
    "mfd_topk_logz_workspace": (c_size, [c_i64, c_i64, c_i64]),
    "mfd_topk_logz": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_int, c_vp, c_vp, c_size, c_vp,
                              c_i64, c_vp]),
    "mfd_topk_logz_static": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_int, c_vp, c_vp]),
    "mfd_build_trees": (c_int, [c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp,
                                c_vp, c_vp, c_vp]),
    "mfd_accept_workspace": (c_size, [c_i64, c_i64]),
    "mfd_accept_tickets": (c_i64, [c_i64, c_i64]),
    "mfd_accept": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_f32, c_vp, c_i64, c_vp, c_vp,
                           c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_size, c_vp, c_i64,
                           c_vp]),
    "mfd_sample_tokens_workspace": (c_size, [c_i64]),
    "mfd_sample_tokens": (c_int, [c_vp, c_i64, c_i64, c_i64, c_f32, c_vp, c_vp, c_vp, c_size, c_vp, c_i64, c_vp]),
    "mfd_follow": (c_int, [c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp,
                           c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mfd_verify_inputs": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                                  c_vp]),
    "mfd_compile_tree": (c_int, [c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                                 c_i64, c_i64, c_i64, c_i64, ctypes.c_uint32, c_vp, c_i64, c_vp]),
    "mfd_tree_attention_workspace": (c_size, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "mfd_tree_attention_tickets": (c_i64, [c_i64, c_i64, c_i64, c_i64]),
    "mfd_tree_attention": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64,
                                   c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_f32, c_i64,
                                   c_vp, c_i64, c_i64, c_i64, c_vp, c_size, c_vp, c_i64, c_vp]),
    "mfd_paged_mode_attention": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64,
                                         c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp,
                                         c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_f32, c_i64, c_vp,
                                         c_i64, c_i64, c_vp, c_size, c_vp, c_i64, c_vp]),
    "mfd_tree_gdn": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64,
                             c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "mfd_tree_gates": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp,
                               c_vp]),
    "mfd_tree_prep": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_f32, c_vp, c_vp,
                              c_vp, c_vp]),
    "mfd_commit_kv_moves": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "mfd_compact_tail": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp,
                                 c_vp]),
    "mfd_gdn_commit": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                               c_vp]),
    "mfd_conv_commit": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp]),
}

MFD_F32, MFD_BF16, MFD_I32, MFD_I64 = 0, 1, 2, 3


def exported_symbols() -> list[str]:
    return list(_SIGS)


def load(build_if_missing: bool = True):
    """Load (building if needed) the library and bind its entry points.  Needs no GPU."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            if not build_if_missing:
                raise RuntimeError(f"{LIB_PATH} is not built; run python -m mfd_b200.build")
            from . import build as _build

            _build.build()
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def lib():
    return _lib if _lib is not None else load()


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().mfd_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("mfd_b200 needs a CUDA device (no CPU fallback)")
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("mfd_b200: expected CUDA tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("mfd_b200: tensors on different devices")
    return dev if dev is not None else torch.device("cuda", torch.cuda.current_device())


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class Workspace:
    """Per-device, per-purpose scratch, grown on demand, plus one per-device ticket buffer.  Tickets live only in
    the ticket buffer, which starts zeroed and which every ticketed kernel leaves zeroed; scratch needs no
    initialisation.  Calls that share them must be ordered on one stream (as the current-stream launches are)."""

    _cache: dict = {}

    @classmethod
    def tickets(cls, device: torch.device, n: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), "__tickets__")
        buf = cls._cache.get(key)
        if buf is None or buf.numel() < n:
            size = max(int(n), 1024)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.int32, device=device)
            cls._cache[key] = buf
        return buf

    @classmethod
    def get(cls, device: torch.device, purpose: str, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), purpose)
        buf = cls._cache.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(int(nbytes), 256)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            cls._cache[key] = buf
        return buf
