"""ctypes binding of the FlashHead CUDA library (include/flashhead.h).

The library is built in-tree (``flash-head_b200/build.py``) next to this
file. There is no CPU fallback: if the library is missing or fails to load,
every FlashHead operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libflashhead_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

FH_OK = 0
FH_ERR_INVALID_ARGUMENT = 1
FH_ERR_CUDA = 2
FH_ERR_WORKSPACE = 3
FH_ERR_UNSUPPORTED = 4

FH_FLAG_NO_FUSED = 1
FH_FLAG_TEST_TIMEOUT = 2

FH_BF16 = 0
FH_FP16 = 1
FH_FP8_E4M3 = 2
FH_FP32 = 3

_STATUS_NAMES = {1: "invalid argument", 2: "CUDA error", 3: "workspace too small",
                 4: "unsupported"}


class FlashHeadError(RuntimeError):
    """A FlashHead C-ABI call returned a non-zero status."""

    def __init__(self, func: str, status: int, message: str):
        super().__init__(f"{func} failed ({_STATUS_NAMES.get(status, status)}): {message}")
        self.status = status


class HeadDesc(ctypes.Structure):
    """Mirror of ``fh_head_desc``."""

    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("n_clusters", ctypes.c_int32),
        ("cluster_size", ctypes.c_int32),
        ("n_probes", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("score_dtype", ctypes.c_int32),
        ("sample_dtype", ctypes.c_int32),
        ("n_special", ctypes.c_int32),
        ("cluster_base", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("w_perm", ctypes.c_void_p),
        ("vocab_map", ctypes.c_void_p),
        ("cluster_w", ctypes.c_void_p),
        ("cluster_scale", ctypes.c_void_p),
        ("centroid_w", ctypes.c_void_p),
        ("centroid_scale", ctypes.c_void_p),
        ("special_slots", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
_U64 = ctypes.c_uint64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "fh_version": (_I, []),
    "fh_last_error": (ctypes.c_char_p, []),
    "fh_head_create": (_I, [ctypes.POINTER(HeadDesc), ctypes.POINTER(_P)]),
    "fh_head_destroy": (_I, [_P]),
    "fh_workspace_bytes": (_SZ, [_P, _I]),
    "fh_workspace_error_offset": (_SZ, []),
    "fh_step_kernel_count": (_I, [_P, _I, _I]),
    "fh_get_next_token": (_I, [_P, _P, _I, _P, _P, _SZ, _P]),
    "fh_get_next_token_noalloc": (_I, [_P, _P, _I, _P, _P]),
    "fh_get_next_token_host": (_I, [_P, _P, _I, _P, _P, _SZ, _P]),
    "fh_workspace_bytes_host": (_SZ, [_P, _I]),
    "fh_get_next_token_sample": (_I, [_P, _P, _I, _F, _U64, _U64, _P, _P, _SZ, _P]),
    "fh_top_clusters": (_I, [_P, _P, _I, _I, _F, _U64, _U64, _P, _P, _P, _SZ, _P]),
    "fh_cluster_scores": (_I, [_P, _P, _I, _I, _F, _U64, _U64, _P, _P]),
    "fh_stage2_next_token": (_I, [_P, _P, _I, _P, _I, _F, _U64, _U64, _P, _P, _SZ, _P]),
    "fh_dense_next_token": (_I, [_P, _P, _I, _I, _F, _U64, _U64, _P, _P, _SZ, _P]),
    "fh_block_sparse_logits": (_I, [_P, _I, _I, _P, _P, _I, _I, _I, _I, _P, _P]),
    "fh_block_sparse_logits_argmax": (_I, [_P, _I, _I, _P, _P, _I, _P, _I, _I, _I, _P, _P, _P]),
    "fh_block_sparse_argmax_atomic": (_I, [_P, _I, _I, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "fh_tp_local_candidates": (_I, [_P, _P, _I, _I, _F, _U64, _U64, _P, _P, _SZ, _P]),
    "fh_tp_select_and_score": (_I, [_P, _P, _I, _I, _P, _I, _F, _U64, _U64, _P, _P, _SZ, _P]),
    "fh_tp_finalize": (_I, [_P, _I, _P, _P]),
    "fh_spec_accept": (_I, [_P, _P, _P, _P, _I, _I, ctypes.c_int32, _P, _P]),
}

_lib = None
_lock = threading.Lock()


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"FlashHead CUDA library not found at {path}; build it with "
                "`python flash-head_b200/build.py` (there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load_library().fh_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Call an fh_* function that returns a status; raise FlashHeadError on failure."""
    st = getattr(load_library(), name)(*args)
    if st != FH_OK:
        raise FlashHeadError(name, st, last_error())


def dtype_code(dtype) -> int:
    import torch
    codes = {torch.bfloat16: FH_BF16, torch.float16: FH_FP16,
             torch.float8_e4m3fn: FH_FP8_E4M3, torch.float32: FH_FP32}
    if dtype not in codes:
        raise ValueError(f"unsupported dtype {dtype}")
    return codes[dtype]


def stream_ptr(stream=None) -> int:
    """Raw cudaStream_t of a torch stream (default: the current stream)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)
