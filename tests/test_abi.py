"""The C ABI library (no GPU needed): it loads, exports every function include/convrot.h declares, and rejects bad
arguments with the documented status codes before touching the device."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "convrot.h")


@pytest.fixture(scope="module")
def lib():
    from hyperflow_h3_flash_b200 import build

    try:
        build.build()
    except (RuntimeError, OSError) as e:  # pragma: no cover - no toolkit
        pytest.skip(f"cannot build libconvrot.so: {e}")
    from hyperflow_h3_flash_b200 import _lib

    return _lib


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(convrot_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_function_is_exported_and_bound(lib):
    names = declared_functions()
    assert len(names) >= 10
    handle = ctypes.CDLL(os.path.join(ROOT, "hyperflow_h3_flash_b200", "libconvrot.so"))
    for name in names:
        assert hasattr(handle, name), name
    assert sorted(lib.SIGNATURES) == names  # the Python binding covers exactly the header


def test_status_strings_and_version(lib):
    L = lib.lib()
    for code in range(8):
        assert L.convrot_status_string(code)
    assert L.convrot_status_string(99) == b"unknown status"
    assert L.convrot_version() >= 100


def test_bad_arguments_are_rejected_before_any_device_call(lib):
    L = lib.lib()
    # group 32 is not a power of 4; group 128 is what the reference rejects too (int8.py:107-108)
    for group in (2, 32, 128, 512):
        rc = L.convrot_rotate_quant(None, 1024, 10, 1024, group, 0, None, 1024, None, None, 0, 0, None, 0, None)
        assert rc == lib.ERR_GROUP
    # K not a multiple of the group
    assert L.convrot_rotate_quant(None, 1040, 10, 1040, 256, 0, None, 1040, None, None, 0, 0, None, 0,
                                  None) == lib.ERR_SHAPE
    # unknown rounding mode
    assert L.convrot_rotate_quant(None, 1024, 10, 1024, 256, 7, None, 1024, None, None, 0, 0, None, 0,
                                  None) == lib.ERR_ARG
    # M == 0 is an empty, successful call
    assert L.convrot_rotate_quant(None, 1024, 0, 1024, 256, 0, None, 1024, None, None, 0, 0, None, 0,
                                  None) == lib.OK
    assert L.convrot_gemm(None, 64, None, 64, None, None, None, None, 0, None, 0, 0, 0, 8, 64, None, 8,
                          None) == lib.OK
    # null operands, misaligned leading dimensions, K % 16, rank above the fused limit
    assert L.convrot_gemm(None, 64, None, 64, None, None, None, None, 0, None, 0, 0, 4, 8, 64, None, 8,
                          None) == lib.ERR_ARG
    p = ctypes.c_void_p(4096)
    assert L.convrot_gemm(p, 72, p, 64, p, p, None, None, 0, None, 0, 0, 4, 8, 64, p, 8, None) == lib.ERR_ALIGN
    assert L.convrot_gemm(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 8, 40, p, 8, None) == lib.ERR_SHAPE
    assert L.convrot_gemm(p, 64, p, 64, p, p, None, p, 320, p, 320, 320, 4, 8, 64, p, 8, None) == lib.ERR_SHAPE
    assert L.convrot_lowrank_down(p, 64, p, 64, 4, 64, 300, p, 304, None) == lib.ERR_SHAPE


def test_workspace_size(lib):
    """The size convrot_linear checks: q rows padded to 16 bytes, xa rows to 8 elements, each part 256-aligned."""
    L = lib.lib()
    a256 = lambda n: -(-n // 256) * 256  # noqa: E731
    for M, K, r in [(333, 5120, 32), (17, 5120, 33), (5, 1040, 4), (1000, 4096, 12), (64, 1024, 0)]:
        ldq, ldxa = -(-K // 16) * 16, -(-r // 8) * 8
        assert L.convrot_workspace_size(M, K, r) == a256(M * ldq) + a256(M * 4) + a256(M * ldxa * 2), (M, K, r)
    assert L.convrot_workspace_size(-1, 5120, 32) == 0


def test_status_mapping_to_exceptions(lib):
    with pytest.raises(ValueError, match="group"):
        lib.check(lib.ERR_GROUP, "x")
    with pytest.raises(lib.ConvrotError):
        lib.check(lib.ERR_TIMEOUT, "x")
    lib.check(lib.OK, "x")


def test_fused_and_exchange_entry_points_reject_bad_arguments(lib):
    """The SwiGLU, gated-residual, AdaLN, scatter / gather and peer entry points check their arguments first."""
    L = lib.lib()
    p = ctypes.c_void_p(4096)
    P = ctypes.c_void_p
    # SwiGLU: N must split into 64-column a/g block pairs
    assert L.convrot_gemm_swiglu(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 96, 64, p, 48, None) == \
        lib.ERR_SHAPE
    # gated residual: residual rows narrower than N, a misaligned pitch, no residual at all
    assert L.convrot_gemm_residual(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 64, 64, p, 32, None, 0,
                                   None, p, 64, None) == lib.ERR_SHAPE
    assert L.convrot_gemm_residual(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 64, 64, p, 68, None, 0,
                                   None, p, 64, None) == lib.ERR_ALIGN
    assert L.convrot_gemm_residual(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 64, 64, None, 64, None, 0,
                                   None, p, 64, None) == lib.ERR_ARG
    # AdaLN prologue: group 256 only, K a multiple of 256 up to 8192, a finite non-negative eps
    args = dict(x=p, ldx=512, M=4, K=512, group=256, rounding=0, sc=p, sh=p, idx=p, ldm=512, eps=1e-6, q=p, ldq=512,
                s=p, h=None, ldh=0)

    def adaln(**kw):
        a = {**args, **kw}
        return L.convrot_rotate_quant_adaln(a["x"], a["ldx"], a["M"], a["K"], a["group"], a["rounding"], a["sc"],
                                            a["sh"], a["idx"], a["ldm"], a["eps"], a["q"], a["ldq"], a["s"], a["h"],
                                            a["ldh"], None)

    assert adaln(group=64) == lib.ERR_GROUP
    assert adaln(K=640, ldx=640, ldq=640, ldm=640) == lib.ERR_SHAPE
    assert adaln(K=8448, ldx=8448, ldq=8448, ldm=8448) == lib.ERR_SHAPE
    assert adaln(eps=-1.0) == lib.ERR_ARG
    assert adaln(eps=float("nan")) == lib.ERR_ARG
    assert adaln(sc=None) == lib.ERR_ARG
    assert adaln(M=0) == lib.OK
    # the epilogue's silu alone: a non-negative count, non-null 2-byte aligned pointers
    assert L.convrot_silu(p, p, -1, None) == lib.ERR_SHAPE
    assert L.convrot_silu(None, p, 8, None) == lib.ERR_ARG
    assert L.convrot_silu(P(4097), p, 8, None) == lib.ERR_ALIGN
    assert L.convrot_silu(None, None, 0, None) == lib.OK
    # scatter / gather: at least two and at most eight chunks, chunk widths the kernels can address
    outs = (P * 9)(*([4096] * 9))
    # grouped layers: 2 to 8 segments, whole 256-column tiles per low-rank segment, ranks a multiple of 8
    def grouped(r, N, S, xa=p):
        return L.convrot_gemm_grouped(p, 64, p, 64, p, p, None, xa, 64, p, 64, r, 4, N, 64, S, outs, 256, None)

    assert grouped(32, 512, 1) == lib.ERR_ARG
    assert grouped(32, 512 * 9, 9) == lib.ERR_ARG
    assert grouped(32, 384, 2) == lib.ERR_SHAPE  # 192-column segments with a low-rank term
    assert grouped(12, 512, 2) == lib.ERR_SHAPE  # rank 12
    assert grouped(32, 512, 2, xa=None) == lib.ERR_ARG
    assert L.convrot_gemm_scatter(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 256, 64, outs, 1, 128,
                                  None) == lib.ERR_ARG
    assert L.convrot_gemm_scatter(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 288, 64, outs, 9, 32,
                                  None) == lib.ERR_ARG
    assert L.convrot_gemm_scatter(p, 64, p, 64, p, p, None, None, 0, None, 0, 0, 4, 96, 64, outs, 2, 48,
                                  None) == lib.ERR_SHAPE  # 48-column chunks
    assert L.convrot_rotate_quant_gather(outs, 2, 192, 4, 384, 256, 0, p, 384, p, None, 0, None) == lib.ERR_SHAPE
    assert L.convrot_rotate_quant_gather(outs, 1, 512, 4, 512, 256, 0, p, 512, p, None, 0, None) == lib.ERR_ARG
    # peer signalling: at most eight ranks, word-aligned flags
    slots = (P * 2)(4096, 4098)
    assert L.convrot_peer_signal(slots, 2, 1, None) == lib.ERR_ARG
    assert L.convrot_peer_signal(slots, 9, 1, None) == lib.ERR_ARG
    assert L.convrot_peer_wait(P(4098), 2, 1, None) == lib.ERR_ARG
    assert L.convrot_ipc_open(None, None) == lib.ERR_ARG
    assert L.convrot_ipc_close(None) == lib.ERR_ARG
