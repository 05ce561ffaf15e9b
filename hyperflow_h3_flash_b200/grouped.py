"""Layers that read one input -- an attention block's to_q / to_k / to_v, a cross-attention's to_k / to_v -- as ONE GEMM
launch.

The reference runs one ``Int8RotLinear`` per projection (transformer.py:197-203) and shares only their quantisation
(``keep_input``, int8.py:150-159).  ``GroupedInt8RotLinear`` also shares the launch.
- The layers' weights are stacked along N.
- The GEMM epilogue writes each layer's columns to that layer's own output tensor.
- The low-rank terms use one down projection over the stacked down weights; each layer's up weights read that
  layer's own xa columns (``convrot_gemm_grouped``).
Outputs are bitwise those of the separate layers.

At small M (config 5's 256 or 333 text tokens) one GEMM fills only a fraction of the SM pairs, and every launch pays
its fixed start-up.  The grouped launch covers all the layers' tiles in one persistent grid.  At large M it saves
the launches' ramp-up and tail.

The group keeps stacked copies of the layers' weights (the layers stay the source of truth).  The copies are rebuilt
when any layer parameter is replaced, moved or modified in place.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from .int8 import _MIN_KERNEL_ROWS, Int8RotLinear, _kernels, _rows


class GroupedInt8RotLinear(nn.Module):
    """``(layer_0(x), ..., layer_{S-1}(x))`` for 2 to 8 ``Int8RotLinear`` layers with the same input width, group,
    output width, rank and bias presence, computed by one quantisation, one down projection and one GEMM launch on
    CUDA (each layer on its own on CPU, as the reference does).

    The layers are held, not registered: the group adds no state of its own to a model's state dict.
    """

    def __init__(self, *layers: Int8RotLinear) -> None:
        super().__init__()
        if not 2 <= len(layers) <= 8 or any(not isinstance(layer, Int8RotLinear) for layer in layers):
            raise ValueError("GroupedInt8RotLinear takes 2 to 8 Int8RotLinear layers")
        first = layers[0]
        for layer in layers[1:]:
            same = (layer.in_features, layer.out_features, layer.group, layer.rank, layer.bias is None) == (
                first.in_features, first.out_features, first.group, first.rank, first.bias is None)
            if not same:
                raise ValueError("grouped layers need the same in/out widths, group, rank and bias presence")
        if first.rank and (first.rank % 8 or first.out_features % 256):
            raise ValueError("grouped low-rank layers need rank % 8 == 0 and out_features % 256 == 0")
        if not first.rank and first.out_features % 32:
            raise ValueError("grouped layers need out_features % 32 == 0")
        self._layers = tuple(layers)
        self.in_features, self.out_features, self.group = first.in_features, first.out_features, first.group
        self.rank = first.rank
        self._cache: tuple | None = None

    @property
    def layers(self) -> tuple[Int8RotLinear, ...]:
        return self._layers

    def _stacked(self) -> dict[str, Tensor | None]:
        params = [p for layer in self._layers for p in layer.parameters()]
        # inference tensors (`torch.inference_mode`) have no version counter: their address alone keys them
        key = tuple((p.device, p.data_ptr(), None if p.is_inference() else p._version) for p in params)
        if self._cache is None or self._cache[0] != key:
            with torch.no_grad():
                def cat(ts):
                    return torch.cat([t.detach() for t in ts])

                stacked = {
                    "qweight": cat(layer.qweight for layer in self._layers),
                    "wscale": cat(layer.wscale for layer in self._layers),
                    "bias": None if self._layers[0].bias is None else cat(layer.bias for layer in self._layers),
                    "down": cat(layer.down.weight for layer in self._layers) if self.rank else None,
                    "up": cat(layer.up.weight for layer in self._layers) if self.rank else None,
                }
            self._cache = (key, stacked)
        return self._cache[1]

    def forward(self, x: Tensor) -> tuple[Tensor, ...]:
        if not x.is_cuda:
            return tuple(layer(x) for layer in self._layers)
        shape = x.shape
        x2 = _rows(x, self.in_features)
        kernels = _kernels()
        Int8RotLinear._last_input.clear()
        if x2.shape[0] >= _MIN_KERNEL_ROWS:
            xq, sx = kernels.rotate_quant(x2, self.group)
        else:
            xq, sx = kernels.rotate_quant_torch_rounding(x2, self.group)
        st = self._stacked()
        xa = kernels.lowrank_down(x2, st["down"]) if self.rank else None
        outs = kernels.convrot_matmul(xq, st["qweight"], sx, st["wscale"], bias=st["bias"], xa=xa, up=st["up"],
                                      segments=len(self._layers))
        return tuple(o.reshape(*shape[:-1], self.out_features).to(x.dtype) for o in outs)


__all__ = ["GroupedInt8RotLinear"]
