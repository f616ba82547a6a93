"""ctypes binding of the C ABI in include/talos_cuda.h (libtalos_cuda.so).

The library is built in-tree by ``talos_b200.build`` (nvcc, sm_100a). There is
no CPU fallback: if the library is missing, loading it raises.
"""
from __future__ import annotations

import ctypes as C
import os

from .build import CUDA_LIB

OK, INVALID_ARG, OOM, CUDA, NCCL, TIMEOUT, OOB, STATE, UNSUPPORTED = range(9)
STEP_AUTO, STEP_FUSED, STEP_LAYERED = range(3)
KV_F32, KV_F16 = range(2)
STATUS_NAMES = ["OK", "INVALID_ARG", "OOM", "CUDA", "NCCL", "TIMEOUT", "OOB", "STATE", "UNSUPPORTED"]


class TalosError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else status}: {msg}")
        self.status = status


class Cfg(C.Structure):
    """``talos_cfg`` == ``Config`` (src/model/config.rs:14-25)."""

    _fields_ = [(n, C.c_uint32) for n in (
        "n_layer", "n_head", "n_head_kv", "n_embd", "n_ff", "context_length", "vocab_size",
        "rope_dim")] + [("rms_eps", C.c_float), ("rope_freq_base", C.c_float)]


# Every symbol include/talos_cuda.h declares, with its ctypes signature.
_vp, _sz, _u32, _i = C.c_void_p, C.c_size_t, C.c_uint32, C.c_int
SIGNATURES = {
    "talos_last_error": (C.c_char_p, []),
    "talos_device_count": (_i, [C.POINTER(_i)]),
    "talos_ctx_create": (_i, [C.POINTER(Cfg), _i, C.POINTER(_vp)]),
    "talos_ctx_create_tp": (_i, [C.POINTER(Cfg), _i, _i, _i, _vp, C.POINTER(_vp)]),
    "talos_nccl_unique_id": (_i, [_vp]),
    "talos_ctx_tp_resync": (_i, [_vp]),
    "talos_ctx_destroy": (_i, [_vp]),
    "talos_weight_upload": (_i, [_vp, C.c_char_p, _vp, _sz, _i, _sz, _sz]),
    "talos_ctx_set_step_kernel": (_i, [_vp, _i]),
    "talos_ctx_step_kernel": (_i, [_vp, C.POINTER(_i)]),
    "talos_ctx_set_kv_dtype": (_i, [_vp, _i]),
    "talos_ctx_set_batch": (_i, [_vp, _i]),
    "talos_forward_batch": (_i, [_vp, C.POINTER(C.c_uint32), C.POINTER(_sz), _i, C.POINTER(C.c_float)]),
    "talos_prefill_slot": (_i, [_vp, _i, C.POINTER(C.c_uint32), _sz, _sz, C.POINTER(C.c_float)]),
    "talos_generate_batch_greedy": (_i, [_vp, C.POINTER(C.c_uint32), C.POINTER(_sz), _i, _sz,
                                         C.POINTER(C.c_uint32)]),
    "talos_ctx_kv_dtype": (_i, [_vp, C.POINTER(_i)]),
    "talos_ctx_device_bytes": (_i, [_vp, C.POINTER(_sz)]),
    "talos_ctx_stream": (_i, [_vp, C.POINTER(_vp)]),
    "talos_cap_context": (_i, [_vp, _sz]),
    "talos_kv_reset": (_i, [_vp]),
    "talos_forward": (_i, [_vp, _u32, _sz, _vp]),
    "talos_forward_hidden": (_i, [_vp, _u32, _sz, _vp]),
    "talos_generate_greedy": (_i, [_vp, _u32, _sz, _sz, _vp]),
    "talos_prefill": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "talos_perplexity": (_i, [_vp, _vp, _sz, C.POINTER(C.c_float), C.POINTER(C.c_double), C.POINTER(_sz)]),
    "talos_profile_step": (_i, [_vp, _u32, _sz, _vp, _vp]),
    "talos_profile_phases": (_i, [_vp, _u32, _sz, _vp, _sz, C.POINTER(_i), C.POINTER(_i)]),
    "talos_dequant": (_i, [_i, _vp, _sz, _vp]),
    "talos_argmax": (_i, [_vp, _sz, C.POINTER(C.c_uint32)]),
    "talos_matvec": (_i, [_i, _i, _vp, _sz, _sz, _sz, _vp, _vp]),
    "talos_matvec_resident": (_i, [_vp, C.c_char_p, _i, _vp, _sz, _sz, _sz, _vp, _vp]),
    "talos_weight_create": (_i, [_i, _i, _vp, _sz, _sz, _sz, C.POINTER(_vp)]),
    "talos_weight_destroy": (_i, [_vp]),
    "talos_weight_packed_bytes": (_i, [_vp, C.POINTER(_sz)]),
    "talos_matvec_dev": (_i, [_vp, _vp, _vp, _vp]),
    "talos_matvec_dev_noalloc": (_i, [_vp, _vp, _vp, _vp]),
    "talos_matvec_bench": (_i, [C.POINTER(_vp), _i, _vp, _vp, _i, C.POINTER(C.c_float)]),
}

_lib = None


def lib_path() -> str:
    return os.environ.get("TALOS_CUDA_LIB", CUDA_LIB)


def load() -> C.CDLL:
    """Load libtalos_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python -m talos_b200.build` (nvcc, sm_100a). "
            "The decode path has no CPU fallback.")
    L = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(status: int) -> None:
    if status != OK:
        raise TalosError(status, load().talos_last_error().decode(errors="replace"))
