"""Seeded synthetic inputs of the benchmark configurations (the reference publishes no dataset for this path).

Everything is drawn from ``torch.Generator`` on the CPU, so the bits are the same on every machine:
seeds x = 0, W = 1, bias = 2, A (= down^T) = 3, B (= up^T) = 4, outlier channels = 5.

* ``x ~ N(0, 1)`` bf16 [M, K] with 1 % of the K input channels scaled by 20 (outliers);
* ``W ~ N(0, 0.02)`` [N, K], stored as the reference's checkpoint format: rotated by the block Hadamard in fp64 and
  quantised per output channel, ``qweight = round(W R / wscale)``, ``wscale = amax / 127`` (tests/test_int8.py:31-36);
* ``bias ~ N(0, 0.01)`` bf16 [N]; ``A [K, r]`` and ``B [r, N]`` ~ N(0, 0.01) bf16, held as ``down.weight = A^T``
  [r, K] and ``up.weight = B^T`` [N, r] (LowRankLinear, transformer.py:48-58).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .int8 import regular_hadamard


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def activations(M: int, K: int, *, seed: int = 0, outlier_seed: int = 5, outlier_scale: float = 20.0) -> torch.Tensor:
    x = torch.randn(M, K, generator=_gen(seed), dtype=torch.float32)
    channels = torch.randperm(K, generator=_gen(outlier_seed))[: max(K // 100, 1)]
    x[:, channels] *= outlier_scale
    return x.to(torch.bfloat16)


def quantize_weight(weight: torch.Tensor, group: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The checkpoint recipe: ``qweight = round(W R / wscale)`` with a per-output-channel fp64 scale."""
    N, K = weight.shape
    h = regular_hadamard(group).double()
    rotated = (weight.double().reshape(N, K // group, group) @ h).reshape(N, K)
    wscale = rotated.abs().amax(1) / 127.0
    qweight = (rotated / wscale[:, None]).round().clamp(-127, 127).to(torch.int8)
    return qweight, wscale.float()


@dataclass
class LinearWeights:
    qweight: torch.Tensor  # int8 [N, K]
    wscale: torch.Tensor  # fp32 [N]
    bias: torch.Tensor | None  # bf16 [N]
    down: torch.Tensor | None  # bf16 [r, K]
    up: torch.Tensor | None  # bf16 [N, r]

    def to(self, device) -> "LinearWeights":
        mv = lambda t: None if t is None else t.to(device)  # noqa: E731
        return LinearWeights(mv(self.qweight), mv(self.wscale), mv(self.bias), mv(self.down), mv(self.up))


def linear_weights(K: int, N: int, *, rank: int = 0, bias: bool = True, group: int = 256,
                   seed_offset: int = 0) -> LinearWeights:
    """Weights of one convrot linear; ``seed_offset`` separates the linears of a block."""
    w = torch.randn(N, K, generator=_gen(1 + 10 * seed_offset)) * 0.02
    qweight, wscale = quantize_weight(w, group)
    b = (torch.randn(N, generator=_gen(2 + 10 * seed_offset)) * 0.01).to(torch.bfloat16) if bias else None
    down = up = None
    if rank:
        A = (torch.randn(K, rank, generator=_gen(3 + 10 * seed_offset)) * 0.01).to(torch.bfloat16)
        B = (torch.randn(rank, N, generator=_gen(4 + 10 * seed_offset)) * 0.01).to(torch.bfloat16)
        down, up = A.t().contiguous(), B.t().contiguous()
    return LinearWeights(qweight, wscale, b, down, up)


def load_into(layer, weights: LinearWeights) -> None:
    """Copies ``weights`` into an ``Int8RotLinear`` built with matching ``bias`` / ``rank``."""
    with torch.no_grad():
        layer.qweight.copy_(weights.qweight)
        layer.wscale.copy_(weights.wscale)
        if weights.bias is not None:
            layer.bias.copy_(weights.bias)
        if weights.down is not None:
            layer.down.weight.copy_(weights.down)
            layer.up.weight.copy_(weights.up)
