"""B200-native (sm_100a) INT8 "convrot" linear: a drop-in for the hot path of HyperFlow H3 Flash.

``hyperflow_h3_flash_b200.int8`` mirrors ``hyperflow_h3_flash.int8`` (src/hyperflow_h3_flash/int8.py);
``hyperflow_h3_flash_b200.ulysses`` shards token rows over GPUs with the seq<->head all-to-all around attention;
``libconvrot.so`` (C ABI: include/convrot.h) holds the CUDA kernels.
"""

from .int8 import (
    INT8_GEMMS,
    KERNEL_OPTIONS,
    ROTATE_QUANTS,
    Int8RotLinear,
    hadamard_factors,
    regular_hadamard,
    resolve_int8_gemm,
    set_kernel_options,
)

__all__ = [
    "INT8_GEMMS",
    "KERNEL_OPTIONS",
    "ROTATE_QUANTS",
    "Int8RotLinear",
    "hadamard_factors",
    "regular_hadamard",
    "resolve_int8_gemm",
    "set_kernel_options",
]
