"""ctypes binding of libgk.so, the C ABI declared in include/gk.h.

This replaces the reference's NVRTC/driver-API launcher
(python/kingdom_ai/gpu_runtime.py:179-221, ``CudaModule.launch``): every
kernel launch goes through one exported C function that takes raw device
pointers, sizes and the current PyTorch stream. There is no fallback: if the
library is missing or a call fails, an exception is raised.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libgk.so"

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_uint64 = ctypes.c_uint64
c_double = ctypes.c_double
c_size_t = ctypes.c_size_t


class PuctOptions(ctypes.Structure):
    _fields_ = [("c_puct", c_double), ("dirichlet_epsilon", c_double), ("fpu_enabled", c_int),
                ("fpu_reduction", c_double)]


class PuctBuffers(ctypes.Structure):
    _fields_ = [("needs_eval", c_void_p), ("leaf_bits", c_void_p), ("leaf_value", c_void_p),
                ("policy", c_void_p), ("noise", c_void_p), ("active", c_void_p), ("active_count", c_void_p),
                ("errors", c_void_p), ("leaf", c_void_p), ("root_allow", c_void_p), ("node_visits", c_void_p)]


class PuctResults(ctypes.Structure):
    _fields_ = [("actions", c_void_p), ("visits", c_void_p), ("policy", c_void_p), ("values", c_void_p),
                ("simulations", c_void_p), ("network_evaluations", c_void_p), ("priors", c_void_p),
                ("best_values", c_void_p), ("nodes", c_void_p), ("root_values", c_void_p),
                ("status", c_void_p)]


class NetStruct(ctypes.Structure):
    _fields_ = [("channels", c_int), ("blocks", c_int), ("conv_w", c_void_p), ("conv_b", c_void_p),
                ("head_w", c_void_p), ("head_b", c_void_p), ("pol_w", c_void_p), ("pol_b", c_void_p),
                ("val_w1", c_void_p), ("val_b1", c_void_p), ("val_w2", c_void_p), ("val_b2", c_void_p),
                ("norm", c_int), ("norm_w", c_void_p), ("norm_b", c_void_p), ("head_norm", c_void_p)]


_SIGNATURES = {
    "gk_initial_records": [c_void_p, c_int64, c_int, c_void_p],
    "gk_initial_bits": [c_void_p, c_int64, c_int, c_void_p],
    "gk_play_records": [c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p],
    "gk_encode_records": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    "gk_records_to_bits": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    "gk_bits_to_records": [c_void_p, c_void_p, c_int64, c_void_p],
    "gk_play_bits": [c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p],
    "gk_encode_bits": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    "gk_random_playouts": [c_uint64, c_uint64, c_int64, c_int, c_void_p, c_void_p, c_void_p],
    "gk_gen_positions": [c_uint64, c_uint64, c_int64, c_void_p, c_void_p],
    "gk_puct_buffers": [c_void_p, c_int64, c_int, ctypes.POINTER(PuctBuffers)],
    "gk_puct_begin": [c_void_p, c_int64, c_int, c_void_p, c_void_p],
    "gk_puct_root_tactics": [c_void_p, c_int64, c_int, c_void_p],
    "gk_replay_validate": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p],
    "gk_puct_noise": [c_void_p, c_int64, c_int, c_uint64, c_uint64, c_double, c_void_p],
    "gk_puct_select": [c_void_p, c_int64, c_int, ctypes.POINTER(PuctOptions), c_void_p],
    "gk_puct_hash_eval": [c_void_p, c_int64, c_int, c_void_p],
    "gk_puct_compact": [c_void_p, c_int64, c_int, c_void_p],
    "gk_puct_expand_backup": [c_void_p, c_int64, c_int, ctypes.POINTER(PuctOptions), c_int, c_void_p],
    "gk_puct_finish": [c_void_p, c_int64, c_int, ctypes.POINTER(PuctResults), c_void_p],
    "gk_puct_search_hash": [c_void_p, c_int64, c_int, c_void_p, ctypes.POINTER(PuctOptions),
                            ctypes.POINTER(PuctResults), c_void_p],
    "gk_mma_selftest": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "gk_net_forward": [ctypes.POINTER(NetStruct), c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                       c_void_p, c_void_p],
    "gk_net_evaluate_puct": [ctypes.POINTER(NetStruct), c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p],
}
_SIZE_FUNCTIONS = {
    "gk_puct_workspace_bytes": [c_int64, c_int],
    "gk_net_weight_bytes": [c_int, c_int],
    "gk_net_headfeat_bytes": [c_int64],
}

_lock = threading.Lock()
_lib = None


def library():
    """Load libgk.so once; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise RuntimeError(f"{LIBRARY_PATH} is missing: build it with build_native.py "
                                   "(the CUDA path has no fallback)")
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, args in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = c_int
            for name, args in _SIZE_FUNCTIONS.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = c_size_t
            _lib = lib
        return _lib


def register(name: str, argtypes, restype=c_int):
    """Bind an additional exported function (used by other modules)."""
    fn = getattr(library(), name)
    fn.argtypes = argtypes
    fn.restype = restype
    return fn


def call(name: str, *args) -> None:
    status = getattr(library(), name)(*args)
    if status != 0:
        if status == -22:
            raise ValueError(f"{name}: invalid argument")
        raise RuntimeError(f"{name} failed with CUDA error {status}")


def ptr(tensor: torch.Tensor | None):
    return None if tensor is None else c_void_p(tensor.data_ptr())


def stream_of(device: torch.device):
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(device) -> torch.device:
    resolved = torch.device(device)
    if resolved.type != "cuda":
        raise ValueError("the batched self-play engine requires a CUDA device")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable")
    index = torch.cuda.current_device() if resolved.index is None else resolved.index
    if not 0 <= index < torch.cuda.device_count():
        raise ValueError("CUDA device index is unavailable")
    return torch.device("cuda", index)
