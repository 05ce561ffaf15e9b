"""INT8 W8A8 "convrot" linear on B200 (sm_100a): a drop-in for ``hyperflow_h3_flash.int8``.

Same module API as the reference (src/hyperflow_h3_flash/int8.py): ``Int8RotLinear(in, out, group)`` with the state
``{qweight int8 [N, K], wscale fp32 [N]}``, ``regular_hadamard``, ``hadamard_factors``, ``KERNEL_OPTIONS`` /
``set_kernel_options``, ``resolve_int8_gemm`` and the kernel namespace ``_kernels()`` with
``rotate_quant(x2, group) -> (q, s)`` and ``int8_matmul(a, b, sa, sb) -> bf16``.

What runs on CUDA tensors: the hand-written sm_100a kernels of ``libconvrot.so`` (C ABI, include/convrot.h):

* ``rotate_quant``: exact block-Hadamard rotation, rounded once to fp32, per-token ``s = max(amax, 1e-12) / 127``,
  ``q = rint(y * (1/s))`` (int8.py:194-221);
* ``int8_matmul``: a tcgen05 ``kind::i8`` GEMM with the ``(acc * sa) * sb -> bf16`` epilogue (int8.py:311, 324).

Two optional extensions, off by default so existing checkpoints load unchanged: ``bias=True`` adds a bf16 ``bias``
[N], and ``rank=r`` adds the low-rank correction ``up(down(x))`` of ``LowRankLinear`` (transformer.py:48-58) with
``down.weight`` [r, K] and ``up.weight`` [N, r]. Both are fused into the GEMM epilogue.

Rows: the reference sends CUDA inputs of fewer than ``_MIN_KERNEL_ROWS`` rows through its torch path, whose rotation
is rounded to bf16 and whose codes divide by the scale (int8.py:164-167, 173-179). Here those rows run on the same CUDA
kernels in that rounding mode, so both regimes reproduce the reference's numbers. CPU tensors take the reference's
torch path, as in the reference. There is no other path: if the CUDA library is missing, CUDA inputs raise.
"""

from __future__ import annotations

import ctypes
import functools
from types import SimpleNamespace
from typing import Any, ClassVar

import torch
from torch import Tensor, nn

from . import _lib

#: Run-time kernel choices of the reference; accepted for compatibility. Every choice runs the tcgen05 kernels.
INT8_GEMMS = ("auto", "triton", "cublas", "sgl", "bf16")
ROTATE_QUANTS = ("dense", "factored")

#: Inputs with fewer rows reproduce the reference's torch-path rounding (int8.py:41-43, 164).
_MIN_KERNEL_ROWS = 17

#: Largest low-rank width fused into the GEMM epilogue (streamed through it in chunks of 64; the reference pads
#: ranks to multiples of 64 at load, transformer.py:45, 205-216).
MAX_FUSED_RANK = 256

KERNEL_OPTIONS: dict[str, Any] = {"int8_gemm": "auto", "rotate_quant": "dense"}


def set_kernel_options(*, int8_gemm: str | None = None, rotate_quant: str | None = None) -> None:
    """Validates and records the reference's kernel options (int8.py:49-57); they do not change the arithmetic."""
    if int8_gemm is not None:
        if int8_gemm not in INT8_GEMMS:
            raise ValueError(f"int8_gemm must be one of {INT8_GEMMS}, got {int8_gemm!r}")
        KERNEL_OPTIONS["int8_gemm"] = int8_gemm
    if rotate_quant is not None:
        if rotate_quant not in ROTATE_QUANTS:
            raise ValueError(f"rotate_quant must be one of {ROTATE_QUANTS}, got {rotate_quant!r}")
        KERNEL_OPTIONS["rotate_quant"] = rotate_quant


def resolve_int8_gemm(device: torch.device) -> str:
    """The GEMM that runs on ``device``: always the sm_100a tcgen05 kernel (int8.py:85-97 picks among backends)."""
    return "tcgen05"


@functools.cache
def regular_hadamard(group: int) -> Tensor:
    """``kron(H4/2, ..., H4/2)`` of size ``group`` (a power of 4), fp32: orthonormal, symmetric, rows sum to one
    (int8.py:100-109). Raises ``ValueError`` for other sizes."""
    h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float64) / 2
    h, n = torch.ones(1, 1, dtype=torch.float64), 1
    while n < group:
        h, n = torch.kron(h, h4), n * 4
    if n != group:
        raise ValueError(f"Hadamard group {group} is not a power of 4")
    return h.float()


def hadamard_factors(group: int) -> tuple[int, int] | None:
    """Split of a group of 2^n channels (n even, group >= 256) into Hadamard sizes ``GA = 4^floor(n/4)`` and
    ``GB = group / GA``, both 16 or more, whose Kronecker product is the group's matrix; ``None`` for any other
    group (the factored rotation's precondition, int8.py:112-119)."""
    n = group.bit_length() - 1
    if group < 256 or group != 1 << n or n % 2:
        return None
    ga = 4 ** (n // 4)
    return ga, group // ga


@functools.cache
def _rotation(group: int, device: torch.device) -> Tensor:
    return regular_hadamard(group).to(device=device, dtype=torch.bfloat16)


class Int8RotLinear(nn.Module):
    """W8A8 linear ``y = (q(x R) @ qweight^T) * s_x * wscale [+ bias] [+ up(down(x))]``, ``R = blockdiag(H_group)``.

    The reference's constructor and state are unchanged (int8.py:127-148); ``bias`` and ``rank`` are keyword-only
    extensions. Linears that read one input (``to_q``, ``to_k``, ``to_v``) quantise it once: a layer with
    ``keep_input = True`` leaves its quantised input for the next layer, which reuses it if it receives the exact
    same, unmodified tensor (int8.py:130-159).
    """

    _last_input: ClassVar[dict[str, Any]] = {}

    def __init__(self, in_features: int, out_features: int, group: int, *, bias: bool = False,
                 rank: int = 0) -> None:
        super().__init__()
        if in_features % group:
            raise ValueError(f"in_features {in_features} is not a multiple of the Hadamard group {group}")
        self.in_features, self.out_features, self.group = in_features, out_features, group
        self.keep_input = False
        # Weights are registered as frozen nn.Parameters rather than buffers, so that offloading hooks which move a
        # module's parameters between host and device treat them like every other weight of the model.
        self.qweight = nn.Parameter(torch.zeros(out_features, in_features, dtype=torch.int8), requires_grad=False)
        self.wscale = nn.Parameter(torch.ones(out_features, dtype=torch.float32), requires_grad=False)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16), requires_grad=False)
        else:
            self.register_parameter("bias", None)
        self.rank = int(rank)
        if self.rank:
            self.down = nn.Linear(in_features, self.rank, bias=False, dtype=torch.bfloat16)
            self.up = nn.Linear(self.rank, out_features, bias=False, dtype=torch.bfloat16)
            self.down.weight.requires_grad_(False)
            self.up.weight.requires_grad_(False)

    def extra_repr(self) -> str:
        extra = f", bias={self.bias is not None}, rank={self.rank}" if (self.bias is not None or self.rank) else ""
        return f"in_features={self.in_features}, out_features={self.out_features}, group={self.group}{extra}"

    def _quantize(self, x: Tensor, x2: Tensor, kernels: SimpleNamespace) -> tuple[Tensor, Tensor]:
        cache = Int8RotLinear._last_input
        # A tensor made under torch.inference_mode() carries no _version (reading it raises), so it is keyed by
        # identity alone: such tensors cannot be modified in place outside inference mode anyway.
        version = None if x.is_inference() else x._version
        hit = cache.get("x") is x and cache.get("version") == version and cache.get("group") == self.group
        quantized = cache["value"] if hit else kernels.rotate_quant(x2, self.group)
        # a shared low-rank projection of the same input travels with the quantisation (see _lowrank_input)
        self._lowrank_hit = cache.get("lowrank") if hit else None
        cache.clear()
        if self.keep_input:
            cache.update(x=x, version=version, group=self.group, value=quantized)
        return quantized

    def _lowrank_input(self, x2: Tensor, kernels: SimpleNamespace) -> Tensor:
        """``down(x)`` for the fused low-rank term.  Layers joined by ``share_lowrank`` that receive the same input
        (q, k, v) compute ``x . [down_q; down_k; down_v]^T`` once and take their slice, extending the reference's
        shared quantisation (int8.py:150-159) to the low-rank projection.  Call after ``_quantize``: the shared
        result lives in the same cache and dies with it."""
        peers = getattr(self, "_lowrank_peers", None)
        stored, self._lowrank_hit = getattr(self, "_lowrank_hit", None), None
        if not peers or sum(layer.rank for layer in peers) > MAX_FUSED_RANK:  # one down GEMM covers 256 outputs
            return kernels.lowrank_down(x2, self.down.weight)
        if stored is not None and stored[0] is peers:
            fused = stored[1]
        else:
            fused = kernels.lowrank_down(x2, _stacked_down(peers))
        if self.keep_input:
            Int8RotLinear._last_input["lowrank"] = (peers, fused)
        start = 0
        for layer in peers:
            if layer is self:
                break
            start += layer.rank
        return fused[:, start:start + self.rank]

    def forward(self, x: Tensor, *, out_chunks: int | None = None, residual: Tensor | None = None,
                gate: Tensor | None = None, gate_index: Tensor | None = None) -> Tensor:
        """``out_chunks = P`` (CUDA only) returns the output packed for the Ulysses all-to-all: ``[P, M, N / P]``,
        column block j of every row in ``[j]`` (see ``forward_packed`` for the matching input).

        ``residual`` returns ``residual + gate[gate_index] * self(x)`` in bf16 steps, the block's gated residual
        (transformer.py:375, 378), fused into the GEMM epilogue on CUDA."""
        if residual is not None and not x.is_cuda:  # the same bf16 tensor ops, unfused
            y = self.forward(x)
            if gate is not None:
                rows = gate.reshape(-1, self.out_features)
                if gate_index is not None:
                    y = rows.index_select(0, gate_index.reshape(-1)).reshape(y.shape) * y
                else:
                    y = rows[0] * y
            return residual + y
        shape = x.shape
        x2 = _rows(x, self.in_features)
        if x2.is_cuda:
            kernels = _kernels()
            if x2.shape[0] >= _MIN_KERNEL_ROWS:
                xq, sx = self._quantize(x, x2, kernels)
            else:
                Int8RotLinear._last_input.clear()
                self._lowrank_hit = None
                xq, sx = kernels.rotate_quant_torch_rounding(x2, self.group)
            xa = self._lowrank_input(x2, kernels) if self.rank else None
            y = kernels.convrot_matmul(xq, self.qweight, sx, self.wscale, bias=self.bias, xa=xa,
                                       up=self.up.weight if self.rank else None, out_chunks=out_chunks,
                                       residual=residual, gate=gate, gate_index=gate_index)
            if out_chunks:
                return y
        else:
            if out_chunks:
                raise ValueError("packed outputs are produced on CUDA tensors only")
            Int8RotLinear._last_input.clear()
            y = self._forward_torch(x2, _rotation(self.group, x2.device))
            if self.bias is not None:
                y = y + self.bias
            if self.rank:
                y = y + self.up(self.down(x2))
        return y.reshape(*shape[:-1], self.out_features).to(x.dtype)

    def forward_packed(self, xp: Tensor, *, out_chunks: int | None = None) -> Tensor:
        """The layer on an input packed as ``[P, M, K / P]`` -- row m is ``cat(xp[0, m], ..., xp[P-1, m])``, the
        receive buffer of the Ulysses head -> seq all-to-all -- without unpacking it (CUDA only)."""
        if not xp.is_cuda or xp.dim() != 3 or xp.shape[0] * xp.shape[2] != self.in_features:
            raise ValueError(f"expected a CUDA tensor [P, M, {self.in_features} / P], got {tuple(xp.shape)}")
        xp = xp.to(torch.bfloat16).contiguous()
        kernels = _kernels()
        Int8RotLinear._last_input.clear()
        self._lowrank_hit = None
        rows = xp.shape[1]
        rounding = _lib.ROUND_KERNEL if rows >= _MIN_KERNEL_ROWS else _lib.ROUND_TORCH
        xq, sx = kernels.rotate_quant_packed(xp, self.group, rounding)
        xa = kernels.lowrank_down_packed(xp, self.down.weight) if self.rank else None
        return kernels.convrot_matmul(xq, self.qweight, sx, self.wscale, bias=self.bias, xa=xa,
                                      up=self.up.weight if self.rank else None, out_chunks=out_chunks)

    def forward_scatter(self, x: Tensor, out_ptrs: list[int], out_ld: int) -> None:
        """The layer with its output written as column chunks to device addresses (CUDA only): chunk j of each row
        to ``out_ptrs[j]`` (``[M, out_ld]`` rows) -- the seq -> head exchange done by the GEMM, when the addresses are
        the other GPUs' receive buffers."""
        x2 = _rows(x, self.in_features)
        if not x2.is_cuda:
            raise ValueError("forward_scatter runs on CUDA tensors only")
        kernels = _kernels()
        if x2.shape[0] >= _MIN_KERNEL_ROWS:
            xq, sx = self._quantize(x, x2, kernels)
        else:
            Int8RotLinear._last_input.clear()
            self._lowrank_hit = None
            xq, sx = kernels.rotate_quant_torch_rounding(x2, self.group)
        xa = self._lowrank_input(x2, kernels) if self.rank else None
        kernels.convrot_matmul(xq, self.qweight, sx, self.wscale, bias=self.bias, xa=xa,
                               up=self.up.weight if self.rank else None, out_ptrs=out_ptrs, out_ld=out_ld)

    def forward_gather(self, x_ptrs: list[int], rows: int, ldx: int, device: torch.device,
                       out: Tensor | None = None) -> Tensor:
        """The layer on rows gathered from column chunks at device addresses (CUDA only): row m is the concatenation
        over j of row m of ``[rows, ldx]`` at ``x_ptrs[j]`` -- the head -> seq exchange done by the rotate kernel's
        row copies, when the addresses are the other GPUs' buffers.  Returns ``[rows, out_features]``, written into
        ``out`` (bf16, contiguous rows) when given."""
        kernels = _kernels()
        Int8RotLinear._last_input.clear()
        self._lowrank_hit = None
        rounding = _lib.ROUND_KERNEL if rows >= _MIN_KERNEL_ROWS else _lib.ROUND_TORCH
        xq, sx, xg = kernels.rotate_quant_gather(x_ptrs, ldx, rows, self.in_features, self.group, device, rounding)
        xa = kernels.lowrank_down(xg, self.down.weight) if self.rank else None
        up = self.up.weight if self.rank else None
        if out is None:
            return kernels.convrot_matmul(xq, self.qweight, sx, self.wscale, bias=self.bias, xa=xa, up=up)
        return kernels.convrot_matmul(xq, self.qweight, sx, self.wscale, bias=self.bias, xa=xa, up=up, out=out)

    def _forward_torch(self, x2: Tensor, rot: Tensor) -> Tensor:
        """The reference's torch path (int8.py:173-179): the rotation is rounded to bf16 and the codes divide by
        the scale. Used for CPU tensors only."""
        g = self.group
        xr = torch.matmul(x2.reshape(-1, self.in_features // g, g), rot).reshape(x2.shape).float()
        sx = xr.abs().amax(1, keepdim=True).clamp_min(1e-12) / 127.0
        xq = torch.clamp(torch.round(xr / sx), -127, 127)
        acc = xq @ self.qweight.float().t()
        return (acc * sx * self.wscale[None, :]).to(torch.bfloat16)


def _stacked_down(peers: tuple) -> Tensor:
    """``[down_q; down_k; down_v]`` for layers joined by ``share_lowrank``, built once and rebuilt only when one of
    the weights is replaced, moved or modified in place (kept on the first layer, keyed by address and version)."""
    weights = [layer.down.weight for layer in peers]
    key = tuple((w.data_ptr(), None if w.is_inference() else w._version) for w in weights)  # no version: inference
    cached = getattr(peers[0], "_stacked_down_cache", None)
    if cached is None or cached[0] != key:
        with torch.no_grad():
            cached = (key, torch.cat([layer.down.weight.detach() for layer in peers]))
        peers[0]._stacked_down_cache = cached
    return cached[1]


def share_lowrank(*layers: Int8RotLinear) -> None:
    """Let layers that read one input (``to_q``, ``to_k``, ``to_v``) compute their low-rank ``down`` projections in
    one pass over the input.  Sharing works together with ``keep_input`` (set it on all but the last layer), exactly
    as the shared quantisation does; outputs are unchanged."""
    if not layers or any(not isinstance(layer, Int8RotLinear) or not layer.rank for layer in layers):
        raise ValueError("share_lowrank takes Int8RotLinear layers that have a low-rank term")
    if len({layer.in_features for layer in layers}) != 1:
        raise ValueError("layers sharing a low-rank projection must read the same input width")
    peers = tuple(layers)
    for layer in layers:
        layer._lowrank_peers = peers


# ------------------------------------------------------------------------------------------------- kernels


def _stream(t: Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require(t: Tensor, name: str, dtype: torch.dtype, ndim: int) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must be contiguous in its last dimension")


def _padded_k(K: int) -> int:
    return -(-K // 16) * 16


def _rows(x: Tensor, k: int) -> Tensor:
    """``x`` as bf16 rows ``[M, k]``, copied only when its last dimension is not unit-stride: a strided row view (a
    column slice of a wider tensor, e.g. the v part of a fused QKV output) goes to the kernels as it is."""
    x2 = x.reshape(-1, k).to(torch.bfloat16)
    return x2 if x2.stride(-1) == 1 else x2.contiguous()


def _pad_cols(t: Tensor, cols: int) -> Tensor:
    if t.shape[1] == cols and t.stride(0) % 16 == 0 and t.data_ptr() % 16 == 0:
        return t
    out = torch.zeros(t.shape[0], cols, dtype=t.dtype, device=t.device)
    out[:, : t.shape[1]] = t
    return out


def rotate_quant(x: Tensor, group: int, rounding: int = _lib.ROUND_KERNEL) -> tuple[Tensor, Tensor]:
    """``(q int8 [M, K], s fp32 [M])`` of the bf16 rows ``x`` (replaces int8.py:326-344)."""
    _require(x, "x", torch.bfloat16, 2)
    M, K = x.shape
    if K % group:
        raise ValueError(f"K = {K} is not a multiple of the Hadamard group {group}")
    Kp = _padded_k(K)
    xs = _pad_cols(x, Kp) if (Kp != K or x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16) else x
    q = torch.empty(M, Kp, dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    rc = _lib.lib().convrot_rotate_quant(_ptr(xs), xs.stride(0), M, Kp, group, rounding, _ptr(q), Kp, _ptr(s),
                                         None, 0, 0, None, 0, _stream(x))
    _lib.check(rc, "convrot_rotate_quant")
    return (q if Kp == K else q[:, :K]), s


def rotate_quant_packed(xp: Tensor, group: int, rounding: int = _lib.ROUND_KERNEL) -> tuple[Tensor, Tensor]:
    """``rotate_quant`` of the rows of a packed ``[P, M, K / P]`` input (the Ulysses receive layout)."""
    _require(xp, "xp", torch.bfloat16, 3)
    P, M, W = xp.shape
    K = P * W
    xp = xp.contiguous()
    q = torch.empty(M, K, dtype=torch.int8, device=xp.device)
    s = torch.empty(M, dtype=torch.float32, device=xp.device)
    rc = _lib.lib().convrot_rotate_quant_packed(_ptr(xp), W, M, K, group, rounding, _ptr(q), K, _ptr(s),
                                                _stream(xp))
    _lib.check(rc, "convrot_rotate_quant_packed")
    return q, s


def lowrank_down_packed(xp: Tensor, down: Tensor) -> Tensor:
    """``bf16(x . down^T)`` for a packed ``[P, M, K / P]`` input."""
    _require(xp, "xp", torch.bfloat16, 3)
    _require(down, "down", torch.bfloat16, 2)
    P, M, W = xp.shape
    K = P * W
    r = down.shape[0]
    xp = xp.contiguous()
    down = down.contiguous()
    ld = -(-r // 8) * 8
    xa = torch.empty(M, ld, dtype=torch.bfloat16, device=xp.device)
    rc = _lib.lib().convrot_lowrank_down_packed(_ptr(xp), W, _ptr(down), down.stride(0), M, K, r, _ptr(xa), ld,
                                                _stream(xp))
    _lib.check(rc, "convrot_lowrank_down_packed")
    return xa if ld == r else xa[:, :r]


def rotate_quant_gather(x_ptrs: list[int], ldx: int, M: int, K: int, group: int, device: torch.device,
                        rounding: int = _lib.ROUND_KERNEL) -> tuple[Tensor, Tensor, Tensor]:
    """``rotate_quant`` of rows gathered from column chunks at device addresses (possibly other GPUs' memory): row m
    is the concatenation over j of row m of ``[M, ldx]`` at ``x_ptrs[j]`` (``K / len(x_ptrs)`` columns each).  Also
    returns the gathered bf16 rows ``[M, K]`` (what the low-rank down projection reads)."""
    n = len(x_ptrs)
    q = torch.empty(M, K, dtype=torch.int8, device=device)
    s = torch.empty(M, dtype=torch.float32, device=device)
    x = torch.empty(M, K, dtype=torch.bfloat16, device=device)
    ptrs = (ctypes.c_void_p * n)(*x_ptrs)
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    rc = _lib.lib().convrot_rotate_quant_gather(ptrs, n, ldx, M, K, group, rounding, _ptr(q), K, _ptr(s), _ptr(x), K,
                                                stream)
    _lib.check(rc, "convrot_rotate_quant_gather")
    return q, s, x


def rotate_quant_adaln(x: Tensor, group: int, scale: Tensor, shift: Tensor, index: Tensor, eps: float = 1e-6,
                       rounding: int = _lib.ROUND_KERNEL) -> tuple[Tensor, Tensor, Tensor]:
    """``rotate_quant`` of ``h = LN(x) * (1 + scale[index]) + shift[index]`` (bf16 steps, LayerNorm without affine
    parameters), computed inside the kernel; returns ``(q, s, h)``.  ``scale`` / ``shift``: bf16 ``[T, K]``,
    ``index``: ``[M]`` integers in ``[0, T)`` (the reference's ``adaln_indices``, transformer.py:345-348)."""
    _require(x, "x", torch.bfloat16, 2)
    M, K = x.shape
    x = x.contiguous()
    scale = scale.to(torch.bfloat16).contiguous()
    shift = shift.to(torch.bfloat16).contiguous()
    if scale.shape != shift.shape or scale.dim() != 2 or scale.shape[1] != K:
        raise ValueError(f"scale / shift must be [T, {K}], got {tuple(scale.shape)} / {tuple(shift.shape)}")
    index = index.to(device=x.device, dtype=torch.int32).contiguous()
    if index.shape != (M,):
        raise ValueError(f"index must be [{M}], got {tuple(index.shape)}")
    q = torch.empty(M, K, dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    h = torch.empty(M, K, dtype=torch.bfloat16, device=x.device)
    rc = _lib.lib().convrot_rotate_quant_adaln(_ptr(x), K, M, K, group, rounding, _ptr(scale), _ptr(shift),
                                               _ptr(index), K, float(eps), _ptr(q), K, _ptr(s), _ptr(h), K,
                                               _stream(x))
    _lib.check(rc, "convrot_rotate_quant_adaln")
    return q, s, h


def adaln_modulate_quantize(x: Tensor, scale: Tensor, shift: Tensor, index: Tensor, group: int,
                            eps: float = 1e-6) -> Tensor:
    """``h = norm(x) * (1 + scale[index]) + shift[index]`` for the q / k / v projections of a block, with their
    shared quantisation computed in the same pass: returns h (bf16, for the low-rank down projection and anything
    else that reads it) and leaves h's codes and scales in the ``keep_input`` cache, so ``to_q(h)`` (with
    ``keep_input`` set, as the reference sets it for to_q / to_k) quantises nothing.  Call site: chunk_block,
    transformer.py:345-353."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
    rounding = _lib.ROUND_KERNEL if x2.shape[0] >= _MIN_KERNEL_ROWS else _lib.ROUND_TORCH
    q, s, h = _kernels().rotate_quant_adaln(x2, group, scale, shift, index.reshape(-1), eps, rounding)
    h = h.reshape(shape)
    cache = Int8RotLinear._last_input
    cache.clear()
    cache.update(x=h, version=None if h.is_inference() else h._version, group=group, value=(q, s))
    return h


def rotate_quant_torch_rounding(x: Tensor, group: int) -> tuple[Tensor, Tensor]:
    """``rotate_quant`` with the reference torch path's rounding (bf16 rotation, division): int8.py:175-178."""
    return rotate_quant(x, group, _lib.ROUND_TORCH)


def lowrank_down(x: Tensor, down: Tensor) -> Tensor:
    """``bf16(x . down^T)`` [M, r]: ``LowRankLinear.down`` (transformer.py:57-58) on kind::f16 tensor cores."""
    _require(x, "x", torch.bfloat16, 2)
    _require(down, "down", torch.bfloat16, 2)
    M, K = x.shape
    r = down.shape[0]
    if down.shape[1] != K:
        raise ValueError(f"down is {tuple(down.shape)}, expected [r, {K}]")
    Kp = -(-K // 8) * 8
    xs = _pad_cols(x, Kp) if (Kp != K or x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16) else x
    ds = _pad_cols(down.contiguous(), Kp) if (Kp != K or down.data_ptr() % 16) else down.contiguous()
    ld = -(-r // 8) * 8
    xa = torch.empty(M, ld, dtype=torch.bfloat16, device=x.device)
    rc = _lib.lib().convrot_lowrank_down(_ptr(xs), xs.stride(0), _ptr(ds), ds.stride(0), M, Kp, r, _ptr(xa), ld,
                                         _stream(x))
    _lib.check(rc, "convrot_lowrank_down")
    return xa if ld == r else xa[:, :r]


def convrot_matmul(a: Tensor, b: Tensor, sa: Tensor, sb: Tensor, *, bias: Tensor | None = None,
                   xa: Tensor | None = None, up: Tensor | None = None, out_chunks: int | None = None,
                   out_ptrs: list[int] | None = None, out_ld: int | None = None,
                   swiglu: bool = False, residual: Tensor | None = None, gate: Tensor | None = None,
                   gate_index: Tensor | None = None, segments: int | None = None,
                   out: Tensor | None = None) -> Tensor | list[Tensor] | None:
    """``bf16((acc * sa) * sb [+ bias] [+ xa . up^T])``, ``acc = a . b^T`` exact (int8.py:376-390 + extensions).

    ``out_chunks = P`` writes the result packed as ``[P, M, N / P]`` (the Ulysses send layout).  ``out_ptrs`` (device
    addresses, possibly in other GPUs' memory) writes column chunk j as ``[M, out_ld]`` rows at ``out_ptrs[j]`` and
    returns None: the Ulysses exchange done by the GEMM's stores.  ``swiglu`` treats b (and sb, bias, up) as a gated
    projection interleaved in 32-row blocks (``ffn.interleave_rows``) and returns ``h = a * silu(g)``, ``[M, N / 2]``.
    ``residual`` (bf16 ``[M, N]``) returns ``residual + gate[gate_index] * y`` in bf16 steps (``gate`` bf16
    ``[T, N]`` or ``[N]``, optional; ``gate_index`` ``[M]``, optional: row 0 for every token).

    ``segments = S`` treats b (and sb, bias, up) as S layers stacked along N that read the same input, and returns
    their S outputs ``[M, N / S]`` from one launch; ``xa`` is then ``[M, S * r]`` (layer s's down projection in columns
    ``[s r, (s + 1) r)``) and ``up`` ``[N, r]``.

    ``out`` (plain form only: bf16 ``[M, N]``, unit column stride, rows 16-byte aligned) receives the result, which
    is also returned."""
    _require(a, "a", torch.int8, 2)
    _require(b, "b", torch.int8, 2)
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError(f"b is {tuple(b.shape)}, expected [N, {K}]")
    sa = sa.reshape(-1).float().contiguous()
    sb = sb.reshape(-1).float().contiguous()
    if sa.numel() != M or sb.numel() != N:
        raise ValueError("scale sizes do not match the operands")
    Kp = _padded_k(K)
    a_s = _pad_cols(a, Kp)
    b_s = _pad_cols(b.contiguous(), Kp)
    if bias is not None:
        bias = bias.reshape(-1).to(torch.bfloat16).contiguous()
        if bias.numel() != N:
            raise ValueError("bias size does not match N")
    if segments:
        return _grouped_matmul(a_s, b_s, sa, sb, bias, xa, up, segments, M, N, Kp)
    r = 0
    if xa is not None or up is not None:
        if xa is None or up is None:
            raise ValueError("the low-rank term needs both xa and up")
        r = xa.shape[1]
        if up.shape != (N, r):
            raise ValueError(f"up is {tuple(up.shape)}, expected [{N}, {r}]")
        if r > MAX_FUSED_RANK:
            raise ValueError(f"low-rank width {r} exceeds the fused limit {MAX_FUSED_RANK}")
        lr = -(-r // 8) * 8
        xa = _pad_cols(xa.to(torch.bfloat16), lr)
        up = _pad_cols(up.to(torch.bfloat16).contiguous(), lr)
    if residual is not None:
        if swiglu or out_ptrs is not None or out_chunks:
            raise ValueError("a residual goes with one plain [M, N] output")
        ldp = -(-N // 8) * 8  # bf16 rows the epilogue reads must start on 16-byte boundaries

        def rows16(t: Tensor) -> Tensor:
            ok = t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0
            return t if ok else _pad_cols(t, ldp)

        res = rows16(residual.reshape(M, N).to(torch.bfloat16))
        g = None if gate is None else rows16(gate.reshape(-1, N).to(torch.bfloat16))
        gi = None
        if gate_index is not None:
            gi = gate_index.reshape(-1).to(device=a.device, dtype=torch.int32).contiguous()
            if gi.numel() != M or g is None:
                raise ValueError("gate_index needs a gate and one index per row")
        ldy = -(-N // 8) * 8
        y = torch.empty(M, ldy, dtype=torch.bfloat16, device=a.device)
        rc = _lib.lib().convrot_gemm_residual(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                              _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                              up.stride(0) if up is not None else 0, r, M, N, Kp, _ptr(res),
                                              res.stride(0), _ptr(g), g.stride(0) if g is not None else 0, _ptr(gi),
                                              _ptr(y), ldy, _stream(a))
        _lib.check(rc, "convrot_gemm_residual")
        return y if ldy == N else y[:, :N]
    if swiglu:
        if out_ptrs is not None or out_chunks:
            raise ValueError("swiglu writes one plain [M, N / 2] output")
        if N % 64:
            raise ValueError(f"a SwiGLU projection needs N % 64 == 0, got N = {N}")
        ldh = -(-(N // 2) // 8) * 8
        h = torch.empty(M, ldh, dtype=torch.bfloat16, device=a.device)
        rc = _lib.lib().convrot_gemm_swiglu(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                            _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                            up.stride(0) if up is not None else 0, r, M, N, Kp, _ptr(h), ldh,
                                            _stream(a))
        _lib.check(rc, "convrot_gemm_swiglu")
        return h if ldh == N // 2 else h[:, : N // 2]
    if out_ptrs is not None:
        n = len(out_ptrs)
        if n < 2 or N % n or out_ld is None:
            raise ValueError(f"N = {N} does not split into {n} chunks, or out_ld is missing")
        ptrs = (ctypes.c_void_p * n)(*out_ptrs)
        rc = _lib.lib().convrot_gemm_scatter(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                             _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                             up.stride(0) if up is not None else 0, r, M, N, Kp, ptrs, n, out_ld,
                                             _stream(a))
        _lib.check(rc, "convrot_gemm_scatter")
        return None
    if out_chunks:
        if N % out_chunks:
            raise ValueError(f"N = {N} does not split into {out_chunks} chunks")
        W = N // out_chunks
        y = torch.empty(out_chunks, M, W, dtype=torch.bfloat16, device=a.device)
        rc = _lib.lib().convrot_gemm_packed(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                            _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                            up.stride(0) if up is not None else 0, r, M, N, Kp, _ptr(y), W,
                                            _stream(a))
        _lib.check(rc, "convrot_gemm_packed")
        return y
    if out is not None:
        if out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or out.stride(1) != 1 or out.stride(0) % 8 \
                or out.data_ptr() % 16 or out.device != a.device:
            raise ValueError(f"out must be bf16 [{M}, {N}] on {a.device} with unit column stride and 16-byte rows")
        rc = _lib.lib().convrot_gemm(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                     _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                     up.stride(0) if up is not None else 0, r, M, N, Kp, _ptr(out), out.stride(0),
                                     _stream(a))
        _lib.check(rc, "convrot_gemm")
        return out
    ldy = -(-N // 8) * 8
    y = torch.empty(M, ldy, dtype=torch.bfloat16, device=a.device)
    rc = _lib.lib().convrot_gemm(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                 _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                 up.stride(0) if up is not None else 0, r, M, N, Kp, _ptr(y), ldy, _stream(a))
    _lib.check(rc, "convrot_gemm")
    return y if ldy == N else y[:, :N]


def _grouped_matmul(a_s: Tensor, b_s: Tensor, sa: Tensor, sb: Tensor, bias: Tensor | None, xa: Tensor | None,
                    up: Tensor | None, S: int, M: int, N: int, Kp: int) -> list[Tensor]:
    """``convrot_gemm_grouped``: S stacked layers, one launch, S outputs (see ``convrot_matmul(segments=S)``)."""
    if S < 2 or N % S:
        raise ValueError(f"N = {N} does not split into {S} layers")
    Ns = N // S
    r = 0
    if xa is not None or up is not None:
        if xa is None or up is None:
            raise ValueError("the low-rank term needs both xa and up")
        r = up.shape[1]
        if up.shape[0] != N or xa.shape[1] != S * r:
            raise ValueError(f"grouped low-rank operands: xa {tuple(xa.shape)}, up {tuple(up.shape)} for {S} layers")
        if r % 8 or Ns % 256 or r > MAX_FUSED_RANK:
            raise ValueError(f"a grouped low-rank term needs r % 8 == 0 (r = {r}) and N / S % 256 == 0 (N / S = {Ns})")
        xa = _pad_cols(xa.to(torch.bfloat16), S * r)
        up = _pad_cols(up.to(torch.bfloat16).contiguous(), r)
    elif Ns % 32:
        raise ValueError(f"grouped outputs need N / S % 32 == 0, got N / S = {Ns}")
    outs = [torch.empty(M, Ns, dtype=torch.bfloat16, device=a_s.device) for _ in range(S)]
    ptrs = (ctypes.c_void_p * S)(*[o.data_ptr() for o in outs])
    rc = _lib.lib().convrot_gemm_grouped(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), _ptr(sa), _ptr(sb),
                                         _ptr(bias), _ptr(xa), xa.stride(0) if xa is not None else 0, _ptr(up),
                                         up.stride(0) if up is not None else 0, r, M, N, Kp, S, ptrs, Ns, _stream(a_s))
    _lib.check(rc, "convrot_gemm_grouped")
    return outs


def int8_matmul(a: Tensor, b: Tensor, sa: Tensor, sb: Tensor) -> Tensor:
    """``bf16((acc * sa) * sb)`` with ``acc = a . b^T`` (int8.py:376-390)."""
    return convrot_matmul(a, b, sa, sb)


def int8_mm_acc(a: Tensor, b: Tensor) -> Tensor:
    """The raw int32 accumulator ``a . b^T`` of the same tcgen05 GEMM (what ``torch._int_mm`` gives, int8.py:362)."""
    _require(a, "a", torch.int8, 2)
    _require(b, "b", torch.int8, 2)
    M, K = a.shape
    N = b.shape[0]
    Kp = _padded_k(K)
    a_s = _pad_cols(a, Kp)
    b_s = _pad_cols(b.contiguous(), Kp)
    ldc = -(-N // 4) * 4
    acc = torch.empty(M, ldc, dtype=torch.int32, device=a.device)
    rc = _lib.lib().convrot_gemm_acc(_ptr(a_s), a_s.stride(0), _ptr(b_s), b_s.stride(0), M, N, Kp, _ptr(acc), ldc,
                                     _stream(a))
    _lib.check(rc, "convrot_gemm_acc")
    return acc if ldc == N else acc[:, :N]


@functools.cache
def _kernels() -> SimpleNamespace:
    """The kernel namespace the layers call (int8.py:182-398). Raises if ``libconvrot.so`` cannot be loaded."""
    _lib.lib()
    return SimpleNamespace(
        rotate_quant=rotate_quant,
        rotate_quant_torch_rounding=rotate_quant_torch_rounding,
        int8_matmul=int8_matmul,
        convrot_matmul=convrot_matmul,
        lowrank_down=lowrank_down,
        int8_mm_acc=int8_mm_acc,
        rotate_quant_packed=rotate_quant_packed,
        lowrank_down_packed=lowrank_down_packed,
        rotate_quant_gather=rotate_quant_gather,
        rotate_quant_adaln=rotate_quant_adaln,
    )


__all__ = [
    "INT8_GEMMS",
    "KERNEL_OPTIONS",
    "MAX_FUSED_RANK",
    "ROTATE_QUANTS",
    "Int8RotLinear",
    "hadamard_factors",
    "regular_hadamard",
    "resolve_int8_gemm",
    "set_kernel_options",
    "share_lowrank",
]
