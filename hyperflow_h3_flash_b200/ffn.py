"""The feed-forward's gated projection with its SwiGLU fused into the INT8 GEMM epilogue.

The reference's feed-forward (``ChunkedFeedForward``, src/hyperflow_h3_flash/transformer.py:75-99) runs the block's
diffusers ``net``: ``net[0]`` is the gated projection -- ``y = proj(x)`` with ``proj`` a 5120 -> 2 * 13824 linear (an
``Int8RotLinear`` in the int8 checkpoint), then ``a, g = y.chunk(2, -1)`` and ``h = a * silu(g)`` -- and ``net[2]``, the
down projection, reads ``h`` (transformer.py:87-90; the "SwiGLU input, 2 * ffn_dim wide per token", :79).

``SwiGLUInt8`` produces ``h`` from the projection's GEMM directly.  Its B operand is the projection with rows
interleaved in 32-row blocks (``interleave_rows``), so every 64 output columns of a GEMM tile hold 32 columns of
``a`` and the matching 32 of ``g``; the epilogue rounds both to bf16 as the projection's output would be, applies
``a * silu(g)`` in the same bf16 steps torch takes, and stores 32 columns of ``h``.  The ``[M, 2 * ffn_dim]``
projection output is never written, nor read back by a separate activation pass.

Which half is the gate comes from diffusers (absent here): ``gate_first=False`` (the default) takes the first half as
``a`` and the second as ``g``.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import _lib
from .int8 import _MIN_KERNEL_ROWS, Int8RotLinear, _kernels, _rows


def interleave_rows(n: int, gate_first: bool = False) -> Tensor:
    """Row order of the fused projection: rows ``[64 j, 64 j + 32)`` are ``a`` rows ``[32 j, 32 j + 32)`` and rows
    ``[64 j + 32, 64 j + 64)`` the ``g`` rows ``[32 j, 32 j + 32)``; ``n`` (the projection width) must be a
    multiple of 64."""
    if n % 64:
        raise ValueError(f"a fused SwiGLU projection needs a width divisible by 64, got {n}")
    half = n // 2
    a0, g0 = (half, 0) if gate_first else (0, half)
    blocks = torch.arange(half // 32).view(-1, 1) * 32 + torch.arange(32).view(1, -1)  # [half / 32, 32]
    return torch.stack([a0 + blocks, g0 + blocks], dim=1).reshape(n)


def silu_bf16(x: Tensor) -> Tensor:
    """``F.silu`` of a bf16 CUDA tensor computed by the fused SwiGLU epilogue's own silu (its table plus the formula
    for inputs outside it; ``convrot_silu``).  Same bits as torch's ``F.silu``; exists so that the epilogue's silu can
    be checked over every bf16 input."""
    if not x.is_cuda or x.dtype != torch.bfloat16:
        raise ValueError(f"silu_bf16 takes a bf16 CUDA tensor, got {x.dtype} on {x.device}")
    x = x.contiguous()
    y = torch.empty_like(x)
    _lib.check(_lib.lib().convrot_silu(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), x.numel(),
                                       ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)),
               "convrot_silu")
    return y


def swiglu_reference(y: Tensor, gate_first: bool = False) -> Tensor:
    """``a * silu(g)`` on the bf16 projection output, as the unfused modules compute it."""
    a, g = y.chunk(2, dim=-1)
    if gate_first:
        a, g = g, a
    return a * F.silu(g)


class SwiGLUInt8(nn.Module):
    """``net[0]`` of a gated feed-forward around an ``Int8RotLinear`` projection, computed by one fused GEMM.

    Built from a loaded projection (which it keeps for its quantisation, its ``down`` low-rank factor and the CPU
    path); the interleaved copies of ``qweight``, ``wscale``, ``bias`` and ``up.weight`` are buffers of this module.
    """

    def __init__(self, proj: Int8RotLinear, *, gate_first: bool = False) -> None:
        super().__init__()
        self.proj = proj
        self.gate_first = gate_first
        self.out_features = proj.out_features // 2
        perm = interleave_rows(proj.out_features, gate_first).to(proj.qweight.device)
        self.register_buffer("qweight", proj.qweight.detach()[perm].contiguous(), persistent=False)
        self.register_buffer("wscale", proj.wscale.detach()[perm].contiguous(), persistent=False)
        bias = getattr(proj, "bias", None)
        self.register_buffer("bias", None if bias is None else bias.detach()[perm].contiguous(), persistent=False)
        up = proj.up.weight.detach()[perm].contiguous() if proj.rank else None
        self.register_buffer("up", up, persistent=False)

    def forward(self, x: Tensor) -> Tensor:
        proj = self.proj
        shape = x.shape
        x2 = _rows(x, proj.in_features)
        if not x2.is_cuda:
            return swiglu_reference(proj(x), self.gate_first)
        kernels = _kernels()
        if x2.shape[0] >= _MIN_KERNEL_ROWS:
            xq, sx = proj._quantize(x, x2, kernels)
        else:
            Int8RotLinear._last_input.clear()
            proj._lowrank_hit = None
            xq, sx = kernels.rotate_quant_torch_rounding(x2, proj.group)
        xa = proj._lowrank_input(x2, kernels) if proj.rank else None
        h = kernels.convrot_matmul(xq, self.qweight, sx, self.wscale, bias=self.bias, xa=xa, up=self.up,
                                   swiglu=True)
        return h.reshape(*shape[:-1], self.out_features)


__all__ = ["SwiGLUInt8", "interleave_rows", "silu_bf16", "swiglu_reference"]
