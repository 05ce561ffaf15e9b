"""ctypes binding of ``libconvrot.so`` (C ABI: include/convrot.h).

The library is loaded from this package's folder. There is no fallback: if it is missing or fails to load, every
call into the CUDA path raises.
"""

from __future__ import annotations

import ctypes
import functools
import os

from .build import LIB

# Status codes (include/convrot.h).
OK, ERR_SHAPE, ERR_GROUP, ERR_ALIGN, ERR_CUDA, ERR_ARCH, ERR_TIMEOUT, ERR_ARG, ERR_SCRATCH = range(9)
NOALLOC_SCRATCH_BYTES = 16 << 20
ROUND_KERNEL, ROUND_TORCH, ROUND_TRITON = 0, 1, 2

_P, _I, _L, _S, _U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_uint64
_U32 = ctypes.c_uint32
IPC_HANDLE_BYTES = 64

#: Every exported function with its argument types, in header order.
SIGNATURES: dict[str, tuple[list, object]] = {
    "convrot_rotate_quant": ([_P, _L, _L, _L, _I, _I, _P, _L, _P, _P, _L, _L, _P, _L, _P], _I),
    "convrot_lowrank_down": ([_P, _L, _P, _L, _L, _L, _L, _P, _L, _P], _I),
    "convrot_gemm": ([_P, _L, _P, _L, _P, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _P, _L, _P], _I),
    "convrot_gemm_acc": ([_P, _L, _P, _L, _L, _L, _L, _P, _L, _P], _I),
    "convrot_gemm_packed": ([_P, _L, _P, _L, _P, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _P, _L, _P], _I),
    "convrot_rotate_quant_packed": ([_P, _L, _L, _L, _I, _I, _P, _L, _P, _P], _I),
    "convrot_lowrank_down_packed": ([_P, _L, _P, _L, _L, _L, _L, _P, _L, _P], _I),
    "convrot_rotate_quant_adaln": ([_P, _L, _L, _L, _I, _I, _P, _P, _P, _L, ctypes.c_float, _P, _L, _P, _P, _L, _P],
                                   _I),
    "convrot_gemm_residual": ([_P, _L, _P, _L, _P, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _P, _L, _P, _L, _P, _P, _L,
                               _P], _I),
    "convrot_gemm_swiglu": ([_P, _L, _P, _L, _P, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _P, _L, _P], _I),
    "convrot_silu": ([_P, _P, _L, _P], _I),
    "convrot_gemm_grouped": ([_P, _L, _P, _L, _P, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _I, _P, _L, _P], _I),
    "convrot_gemm_scatter": ([_P, _L, _P, _L, _P, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _P, _I, _L, _P], _I),
    "convrot_rotate_quant_gather": ([_P, _I, _L, _L, _L, _I, _I, _P, _L, _P, _P, _L, _P], _I),
    "convrot_ipc_handle": ([_P, _P, _P], _I),
    "convrot_ipc_open": ([_P, _P], _I),
    "convrot_ipc_close": ([_P], _I),
    "convrot_peer_signal": ([_P, _I, _U32, _P], _I),
    "convrot_peer_wait": ([_P, _I, _U32, _P], _I),
    "convrot_copy_blocks": ([_P, _P, _P, _I, _P], _I),
    "convrot_workspace_size": ([_L, _L, _L], _S),
    "convrot_linear": ([_P, _L, _P, _L, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _I, _P, _S, _P, _L, _P], _I),
    "convrot_linear_noalloc": ([_P, _L, _P, _L, _P, _P, _P, _L, _P, _L, _L, _L, _L, _L, _I, _P, _L, _P], _I),
    "convrot_status_string": ([_I], ctypes.c_char_p),
    "convrot_last_cuda_error": ([], _I),
    "convrot_poll_error": ([_P], _I),
    "convrot_set_wait_limit_ns": ([_U64], None),
    "convrot_set_gemm_mode": ([_I], _I),
    "convrot_set_rotate_variant": ([_I], _I),
    "convrot_set_rotate_tuning": ([_I, _I], _I),
    "convrot_version": ([], _I),
    "convrot_split_k_fallbacks": ([], _L),
}


class ConvrotError(RuntimeError):
    """A CUDA-side failure of the convrot library (CUDA error, wrong architecture, expired wait)."""


@functools.cache
def lib() -> ctypes.CDLL:
    """The loaded library; raises if it is absent (build it with ``python -m hyperflow_h3_flash_b200.build``)."""
    if not os.path.exists(LIB):
        raise ConvrotError(f"{LIB} is missing: build it with `python -m hyperflow_h3_flash_b200.build`")
    handle = ctypes.CDLL(LIB)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = res
    return handle


def status_string(code: int) -> str:
    return lib().convrot_status_string(code).decode()


def check(code: int, what: str) -> None:
    """Maps a status to the reference's exception style: ValueError for bad arguments, ConvrotError otherwise."""
    if code == OK:
        return
    message = f"{what}: {status_string(code)}"
    if code in (ERR_SHAPE, ERR_GROUP, ERR_ALIGN, ERR_ARG, ERR_SCRATCH):
        raise ValueError(message)
    if code == ERR_CUDA:
        message += f" (CUDA error {lib().convrot_last_cuda_error()})"
    raise ConvrotError(message)
