"""ctypes bindings of the C ABI (``include/moe_b200.h``) and of the CPU input generator.

The CUDA library is the only compute path: there is no Python or CPU fallback. If
``libmoe_b200.so`` is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_lock = threading.Lock()
_cuda = None
_synth_cpu = None

c_int, c_float, c_size_t, c_void_p, c_uint64 = (ctypes.c_int, ctypes.c_float, ctypes.c_size_t,
                                                 ctypes.c_void_p, ctypes.c_uint64)
c_int_p = ctypes.POINTER(ctypes.c_int)
c_size_t_p = ctypes.POINTER(ctypes.c_size_t)

# name -> (restype, argtypes); every symbol declared in include/moe_b200.h.
CUDA_SIGNATURES = {
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_get_status": (c_int, [c_int_p, c_int]),
    "moe_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "moe_get_wait_limit_ns": (c_int, [ctypes.POINTER(ctypes.c_ulonglong)]),
    "moe_probe_ep_barrier_timeout": (c_int, [c_void_p, c_void_p]),
    "moe_probe_mbar_timeout": (c_int, [c_int, c_void_p, c_void_p]),
    "moe_pack_w13_bytes": (c_size_t, [c_int]),
    "moe_pack_w13": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "moe_pack_w2_bytes": (c_size_t, [c_int]),
    "moe_pack_w2": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "moe_forward_workspace_bytes": (c_size_t, [c_int, c_int]),
    "moe_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_float, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t,
                            c_void_p]),
    "moe_forward_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_float, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t,
                                c_void_p]),
    "moe_shared_expert_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                          c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "moe_forward_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_void_p,
                                    c_void_p]),
    "moe_forward_profiled": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_void_p,
                                     c_void_p, c_size_t, c_void_p, c_void_p]),
    "moe_route": (c_int, [c_void_p, c_void_p, c_float, c_int, c_void_p, c_void_p, c_void_p]),
    "moe_workspace_layout": (c_int, [c_int, c_int, c_size_t_p, c_int]),
    "moe_ep_symmetric_bytes": (c_size_t, [c_int, c_int, c_int]),
    "moe_ep_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "moe_ep_create": (c_int, [c_int, c_int, c_int, c_int, c_void_p, ctypes.POINTER(c_void_p), c_void_p]),
    "moe_ep_connect": (c_int, [c_void_p, c_void_p]),
    "moe_ep_destroy": (c_int, [c_void_p]),
    "moe_ep_info": (c_int, [c_void_p, c_int_p]),
    "moe_ep_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p, c_float, c_int, c_void_p, c_void_p,
                               c_size_t, c_void_p]),
    "moe_ep_forward_profiled": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p, c_float, c_int, c_void_p,
                                        c_void_p, c_size_t, c_void_p, c_void_p]),
    "moe_quantize_hidden": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "moe_gate_packed_bytes": (c_size_t, []),
    "moe_pack_gate": (c_int, [c_void_p, c_void_p, c_void_p]),
    "moe_gate_quantize": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "moe_synth_logits": (c_int, [c_void_p, c_uint64, c_int, c_int, c_void_p, c_void_p]),
    "moe_synth_bias": (c_int, [c_void_p, c_uint64, c_int, c_float, c_void_p, c_int, c_float,
                               c_void_p, c_void_p]),
    "moe_synth_hidden": (c_int, [c_void_p, c_uint64, c_int, c_float, c_void_p, c_void_p, c_void_p]),
    "moe_synth_w13": (c_int, [c_void_p, c_uint64, c_int, c_int, c_float, c_void_p, c_void_p,
                              c_void_p]),
    "moe_synth_w2": (c_int, [c_void_p, c_uint64, c_int, c_int, c_float, c_void_p, c_void_p,
                             c_void_p]),
}

SYNTH_CPU_SIGNATURES = {
    "moe_synth_cpu_logits": (None, [c_void_p, c_uint64, c_int, c_int, c_void_p]),
    "moe_synth_cpu_bias": (None, [c_void_p, c_uint64, c_int, c_float, c_void_p, c_int, c_float,
                                  c_void_p]),
    "moe_synth_cpu_hidden": (None, [c_void_p, c_uint64, c_int, c_float, c_void_p, c_void_p]),
    "moe_synth_cpu_w13": (None, [c_void_p, c_uint64, c_int, c_int, c_float, c_void_p, c_void_p]),
    "moe_synth_cpu_w2": (None, [c_void_p, c_uint64, c_int, c_int, c_float, c_void_p, c_void_p]),
}


def _bind(lib, sigs):
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def cuda_lib():
    """The loaded ``libmoe_b200.so`` (built in-tree on first use if absent)."""
    global _cuda
    with _lock:
        if _cuda is None:
            path = _build.CUDA_LIB
            if not os.path.exists(path):
                _build.build_cuda()
            _cuda = _bind(ctypes.CDLL(path), CUDA_SIGNATURES)
        return _cuda


def synth_cpu_lib():
    global _synth_cpu
    with _lock:
        if _synth_cpu is None:
            path = _build.SYNTH_CPU_LIB
            if not os.path.exists(path):
                _build.build_synth_cpu()
            _synth_cpu = _bind(ctypes.CDLL(path), SYNTH_CPU_SIGNATURES)
        return _synth_cpu


class MoEError(RuntimeError):
    """A failed call of the C ABI (the reference raises RuntimeError from TORCH_CHECK)."""


def check(rc: int) -> None:
    if rc != 0:
        msg = cuda_lib().moe_last_error().decode(errors="replace")
        raise MoEError(msg or f"moe call failed with code {rc}")


# Bits of the device status word (include/moe_b200.h).
ST_TIMEOUT_PRODUCER, ST_TIMEOUT_MMA, ST_TIMEOUT_EPILOGUE, ST_BAD_INDEX, ST_EP_TIMEOUT = 1, 2, 4, 8, 16
EP_HANDLE_BYTES = 64


def device_status(reset: bool = True) -> int:
    """Synchronise and return the kernels' status word (0 = no timeout / bad metadata)."""
    v = ctypes.c_int(0)
    check(cuda_lib().moe_get_status(ctypes.byref(v), 1 if reset else 0))
    return v.value


def set_wait_limit_ns(ns: int) -> None:
    """Limit of every bounded wait in the kernels on the current device (default 2 s)."""
    check(cuda_lib().moe_set_wait_limit_ns(int(ns)))


def wait_limit_ns() -> int:
    v = ctypes.c_ulonglong(0)
    check(cuda_lib().moe_get_wait_limit_ns(ctypes.byref(v)))
    return v.value


def workspace_layout(T: int, E_local: int) -> dict:
    names = ["counts", "dense_base", "topk_idx", "topk_w", "token_nr", "token_route",
             "route_token", "route_w", "a_tiled", "a_scale", "c_hi", "c_lo", "c_scale", "partial",
             "tile_ready", "total"]
    arr = (ctypes.c_size_t * len(names))()
    n = cuda_lib().moe_workspace_layout(T, E_local, arr, len(names))
    if n <= 0:
        check(1)
    return dict(zip(names, list(arr)))
