"""CPU oracle for the INT8 convrot linear -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module, and only as
the checker. The product path (``hyperflow_h3_flash_b200``) never imports it and fails loudly when its CUDA library
is missing.

Two layers:

* ``convrot_oracle.c`` (ctypes): the bit-exact restatement of the reference's kernel arithmetic: exact rotation
  rounded once, scale/inverse, rint, int32 accumulator, and the ``(acc * sa) * sb`` epilogue
  (src/hyperflow_h3_flash/int8.py:194-221, 306-324).
* numpy: ``regular_hadamard`` (int8.py:100-109), ``hadamard_factors`` (int8.py:112-119), the checkpoint recipe
  ``quantize_weight`` (tests/test_int8.py:31-36), the composite reference for the fused bias + low-rank output
  (int8 output + bias + ``up(down(x))``, transformer.py:57-58), and ``forward_cpu_port``, a port of the reference's
  CPU path ``Int8RotLinear._forward_torch`` (int8.py:173-179) on numpy/BLAS, timed as the CPU baseline.

bf16 arrays cross this API as ``np.uint16`` bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from functools import lru_cache

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")


def build() -> str:
    """Compiles ``convrot_oracle.c`` with the Makefile beside it (gcc, pthreads); returns the library path."""
    src = os.path.join(_HERE, "convrot_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


@lru_cache(maxsize=1)
def _lib() -> ctypes.CDLL:
    lib = ctypes.CDLL(build())
    P, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.oracle_rotate.argtypes = [P, L, I, I, I, P, P]
    lib.oracle_rotate_quant.argtypes = [P, L, I, I, I, P, L, P]
    lib.oracle_rotate_quant_cpu.argtypes = [P, L, I, I, I, P, L, P]
    lib.oracle_int8_gemm.argtypes = [P, L, P, L, I, I, I, P, L]
    lib.oracle_epilogue.argtypes = [P, L, P, P, P, P, L, P, L, I, I, I, P, L]
    lib.oracle_epilogue.restype = None
    lib.oracle_lowrank_down.argtypes = [P, L, P, L, I, I, I, P, L]
    lib.oracle_lowrank_down.restype = None
    lib.oracle_f32_to_bf16.argtypes = [P, L, P]
    lib.oracle_f32_to_bf16.restype = None
    lib.oracle_set_threads.argtypes = [I]
    lib.oracle_set_threads.restype = None
    lib.oracle_get_threads.restype = I
    return lib


def set_threads(n: int) -> None:
    """Threads the C oracle uses (0 = all online CPUs)."""
    _lib().oracle_set_threads(int(n))


def get_threads() -> int:
    return int(_lib().oracle_get_threads())


def _ptr(a: np.ndarray | None) -> ctypes.c_void_p | None:
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------------------------------------ bf16 helpers


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _lib().oracle_f32_to_bf16(_ptr(x), x.size, _ptr(out))
    return out


# ---------------------------------------------------------------------------------------- Hadamard (numpy)


def regular_hadamard(group: int) -> np.ndarray:
    """``kron(H4/2, ..., H4/2)`` of size ``group`` (a power of 4), float64 (int8.py:100-109).

    Raises ``ValueError`` for any other size, as the reference does.
    """
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64) / 2
    h, n = np.ones((1, 1)), 1
    while n < group:
        h, n = np.kron(h, h4), n * 4
    if n != group:
        raise ValueError(f"Hadamard group {group} is not a power of 4")
    return h


def hadamard_factors(group: int) -> tuple[int, int] | None:
    """``(GA, GB)`` with ``H_group = kron(H_GA, H_GB)``, both >= 16, or None (int8.py:112-119)."""
    n = group.bit_length() - 1
    if group < 256 or group != 1 << n or n % 2:
        return None
    ga = 4 ** (n // 4)
    return ga, group // ga


# ------------------------------------------------------------------------------ kernel-semantics restatement


def rotate(x_bits: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray, int]:
    """Exact block rotation of bf16 rows: (fp32-rounded y, bf16-rounded y bits, wide-span group count)."""
    x = _c(x_bits, np.uint16)
    M, K = x.shape
    y = np.empty((M, K), np.float32)
    yb = np.empty((M, K), np.uint16)
    rc = _lib().oracle_rotate(_ptr(x), K, M, K, group, _ptr(y), _ptr(yb))
    _check(rc)
    return y, yb, rc


def rotate_quant(x_bits: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """Kernel semantics of ``rotate_quant`` (int8.py:194-221): ``(q int8 [M,K], s fp32 [M])``."""
    x = _c(x_bits, np.uint16)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty((M,), np.float32)
    _check(_lib().oracle_rotate_quant(_ptr(x), K, M, K, group, _ptr(q), K, _ptr(s)))
    return q, s


def rotate_quant_cpu(x_bits: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """CPU-path semantics (int8.py:175-178): bf16-rounded rotation, ``rint(xr / sx)``."""
    x = _c(x_bits, np.uint16)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty((M,), np.float32)
    _check(_lib().oracle_rotate_quant_cpu(_ptr(x), K, M, K, group, _ptr(q), K, _ptr(s)))
    return q, s


def int8_gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact ``a [M,K] . b [N,K]^T`` as int32 (int8.py:306, 362); raises if a sum leaves int32."""
    a = _c(a, np.int8)
    b = _c(b, np.int8)
    M, K = a.shape
    N = b.shape[0]
    acc = np.empty((M, N), np.int32)
    _check(_lib().oracle_int8_gemm(_ptr(a), K, _ptr(b), K, M, N, K, _ptr(acc), N))
    return acc


def epilogue(acc, sa, sb, bias=None, xa=None, B=None) -> np.ndarray:
    """``bf16_rn(((acc * sa) * sb) [+ bias] [+ xa . B])`` as bf16 bits (int8.py:311, 324)."""
    acc = _c(acc, np.int32)
    sa = _c(sa, np.float32)
    sb = _c(sb, np.float32)
    M, N = acc.shape
    bias = None if bias is None else _c(bias, np.uint16)
    r = 0
    if xa is not None:
        xa = _c(xa, np.uint16)
        B = _c(B, np.uint16)
        r = xa.shape[1]
    out = np.empty((M, N), np.uint16)
    _lib().oracle_epilogue(_ptr(acc), N, _ptr(sa), _ptr(sb), _ptr(bias), _ptr(xa), r, _ptr(B), N, r, M, N,
                           _ptr(out), N)
    return out


def lowrank_down(x_bits: np.ndarray, A_bits: np.ndarray) -> np.ndarray:
    """``bf16(x . A)``: the ``down`` projection of ``LowRankLinear`` (transformer.py:57-58), bf16 bits."""
    x = _c(x_bits, np.uint16)
    A = _c(A_bits, np.uint16)
    M, K = x.shape
    r = A.shape[1]
    xa = np.empty((M, r), np.uint16)
    _lib().oracle_lowrank_down(_ptr(x), K, _ptr(A), r, M, K, r, _ptr(xa), r)
    return xa


def convrot_linear(x_bits, qweight, wscale, group, bias=None, A=None, B=None) -> dict:
    """The whole fused op under kernel semantics, with every intermediate (codes, scales, acc, xa, out)."""
    q, s = rotate_quant(x_bits, group)
    acc = int8_gemm(q, qweight)
    xa = lowrank_down(x_bits, A) if A is not None else None
    out = epilogue(acc, s, wscale, bias, xa, B)
    return dict(q=q, s=s, acc=acc, xa=xa, out=out)


def composite_reference(x_bits, qweight, wscale, group, bias=None, A=None, B=None) -> np.ndarray:
    """What the reference's modules compute for the fused op, as bf16 bits:
    ``bf16(bf16(Int8RotLinear(x) + bias) + up(down(x)))`` with ``up(down(x)) = bf16(bf16(x.A).B)``.

    The int8 part uses kernel semantics (the reference's CUDA path); the adds round to bf16 after each step, as
    separate bf16 torch modules do.
    """
    q, s = rotate_quant(x_bits, group)
    acc = int8_gemm(q, qweight)
    y = bf16_to_f32(epilogue(acc, s, wscale))
    if bias is not None:
        y = bf16_to_f32(f32_to_bf16(y + bf16_to_f32(bias)[None, :]))
    if A is not None:
        xa = bf16_to_f32(lowrank_down(x_bits, A)).astype(np.float64)
        lr = bf16_to_f32(f32_to_bf16((xa @ bf16_to_f32(B).astype(np.float64)).astype(np.float32)))
        y = bf16_to_f32(f32_to_bf16(y + lr))
    return f32_to_bf16(y)


def swiglu(y_bits: np.ndarray, gate_first: bool = False) -> np.ndarray:
    """The gated feed-forward activation on a projection's bf16 output, as bf16 bits: ``a, g = y.chunk(2, -1)``
    (``g, a`` with gate_first), ``h = bf16(a * bf16(silu(g)))``, ``silu(g) = g / (1 + exp(-g))`` in fp32 -- the bf16
    torch ops of the gated ``net[0]`` that the reference's ChunkedFeedForward runs (transformer.py:87-90; the module
    itself is diffusers', absent here).  numpy's float32 exp may differ from CUDA's in the last bit, so results can
    differ from a GPU's by one bf16 ulp where silu lands next to a rounding boundary."""
    y = bf16_to_f32(y_bits)
    half = y.shape[-1] // 2
    a, g = (y[..., half:], y[..., :half]) if gate_first else (y[..., :half], y[..., half:])
    with np.errstate(over="ignore"):
        s = (g / (np.float32(1) + np.exp(-g))).astype(np.float32)
    s = bf16_to_f32(f32_to_bf16(s))
    return f32_to_bf16((a * s).astype(np.float32))


def adaln_modulate(x_bits: np.ndarray, scale_bits: np.ndarray, shift_bits: np.ndarray, index: np.ndarray,
                   eps: float = 1e-6) -> np.ndarray:
    """``h = norm1(x) * (1 + scale[idx]) + shift[idx]`` as the reference's chunk_block writes it
    (transformer.py:346-348), each bf16 tensor op rounded to bf16, as bf16 bits.  ``norm1`` is diffusers' module
    (absent here); this restates a LayerNorm without affine parameters: mean and variance of the row in float64,
    ``mean`` and ``1/sqrt(var + eps)`` rounded once to float32, ``(x - mean) * rstd`` in float32."""
    x32 = bf16_to_f32(x_bits)
    x64 = x32.astype(np.float64)
    mean = x64.mean(axis=1)
    var = np.maximum((x64 * x64).mean(axis=1) - mean * mean, 0.0)
    mean_f = mean.astype(np.float32)[:, None]
    rstd_f = (1.0 / np.sqrt(var + np.float64(np.float32(eps)))).astype(np.float32)[:, None]
    n = bf16_to_f32(f32_to_bf16(((x32 - mean_f).astype(np.float32) * rstd_f).astype(np.float32)))
    one_s = bf16_to_f32(f32_to_bf16((np.float32(1) + bf16_to_f32(scale_bits)[index]).astype(np.float32)))
    t = bf16_to_f32(f32_to_bf16((n * one_s).astype(np.float32)))
    return f32_to_bf16((t + bf16_to_f32(shift_bits)[index]).astype(np.float32))


def forward_cpu_port(x_bits: np.ndarray, qweight: np.ndarray, wscale: np.ndarray, group: int,
                     rotation: np.ndarray | None = None) -> np.ndarray:
    """numpy/BLAS port of the reference CPU path ``Int8RotLinear._forward_torch`` (int8.py:173-179).

    Returns bf16 bits. ``xr = bf16(x . H)`` (the reference runs this matmul in bf16), ``sx = max(amax,1e-12)/127``,
    ``xq = rint(xr / sx)`` clamped to +-127, then ``(xq . qweight^T) * sx * wscale`` in fp32 -> bf16.
    """
    M, K = x_bits.shape
    h = (regular_hadamard(group) if rotation is None else rotation).astype(np.float32)
    x = bf16_to_f32(x_bits).reshape(M, K // group, group)
    xr = bf16_to_f32(f32_to_bf16(np.matmul(x, h))).reshape(M, K)
    sx = np.maximum(np.abs(xr).max(axis=1, keepdims=True), np.float32(1e-12)) / np.float32(127.0)
    xq = np.clip(np.rint(xr / sx), -127, 127)
    y = (xq @ qweight.astype(np.float32).T) * sx * wscale[None, :].astype(np.float32)
    return f32_to_bf16(y.astype(np.float32))


def quantize_weight(weight: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """The checkpoint recipe (tests/test_int8.py:31-36): ``qweight = round(W R / wscale)``, per-row fp64 scale."""
    N, K = weight.shape
    h = regular_hadamard(group)
    rotated = (weight.astype(np.float64).reshape(N, K // group, group) @ h).reshape(N, K)
    wscale = np.abs(rotated).max(axis=1) / 127.0
    q = np.clip(np.round(rotated / wscale[:, None]), -127, 127).astype(np.int8)
    return q, wscale.astype(np.float32)


def _check(rc: int) -> None:
    if rc == -1:
        raise ValueError("oracle: non-finite input")
    if rc == -2:
        raise ValueError("oracle: group must be a power of 4 dividing K")
    if rc == -3:
        raise OverflowError("oracle: int8 GEMM sum leaves int32")
