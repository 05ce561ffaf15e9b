"""The fused SwiGLU projection: host logic on CPU (row interleave, CPU path, oracle restatement)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from hyperflow_h3_flash_b200 import ffn
from hyperflow_h3_flash_b200 import int8 as I
from hyperflow_h3_flash_b200 import synthetic
from oracle import oracle as O


def test_interleave_rows_pairs_32_row_blocks_of_each_half():
    perm = ffn.interleave_rows(256)
    assert sorted(perm.tolist()) == list(range(256))
    assert perm[:32].tolist() == list(range(0, 32)) and perm[32:64].tolist() == list(range(128, 160))
    assert perm[64:96].tolist() == list(range(32, 64)) and perm[96:128].tolist() == list(range(160, 192))
    gf = ffn.interleave_rows(256, gate_first=True)
    assert gf[:32].tolist() == list(range(128, 160)) and gf[32:64].tolist() == list(range(0, 32))
    try:
        ffn.interleave_rows(96)
    except ValueError:
        pass
    else:
        raise AssertionError("a width that is not a multiple of 64 must be refused")


def test_cpu_path_is_the_unfused_composition():
    K, N = 512, 256
    w = synthetic.linear_weights(K, N, rank=16, bias=True, group=256)
    proj = I.Int8RotLinear(K, N, 256, bias=True, rank=16)
    synthetic.load_into(proj, w)
    fused = ffn.SwiGLUInt8(proj)
    x = synthetic.activations(24, K, seed=4)
    y = proj(x)
    assert torch.equal(fused(x), y[:, :128] * F.silu(y[:, 128:]))
    assert fused(x).shape == (24, 128)


def test_oracle_swiglu_matches_torch_cpu_within_one_ulp():
    g = torch.Generator().manual_seed(0)
    y = (torch.randn(64, 512, generator=g) * 4).to(torch.bfloat16)
    y[0, :8] = torch.tensor([0.0, -0.0, 100.0, -100.0, -90.0, 88.0, 1e-3, -1e-3])
    ref = ffn.swiglu_reference(y).view(torch.int16).numpy().view(np.uint16)
    got = O.swiglu(y.view(torch.int16).numpy().view(np.uint16))
    diff = np.abs(got.astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() >= 0.999


def test_oracle_adaln_matches_torch_layer_norm_composition_within_one_ulp():
    """The oracle's AdaLN restatement against the bf16 torch ops of chunk_block (transformer.py:346-348) with a
    non-affine LayerNorm on CPU (torch's own statistics: differences of one bf16 ulp where a value sits next to a
    rounding boundary)."""
    g = torch.Generator().manual_seed(1)
    M, K, T = 64, 1024, 3
    x = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16)
    x[:, ::97] *= 30
    scale = (torch.randn(T, K, generator=g) * 0.1).to(torch.bfloat16)
    shift = (torch.randn(T, K, generator=g) * 0.1).to(torch.bfloat16)
    idx = torch.randint(0, T, (M,), generator=g)
    n = F.layer_norm(x, (K,), eps=1e-6)
    ref = n * (1.0 + scale.index_select(0, idx)) + shift.index_select(0, idx)
    u16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    got = O.adaln_modulate(u16(x), u16(scale), u16(shift), idx.numpy())
    assert (got == u16(ref)).mean() >= 0.995
    # t + shift can cancel: bound by one bf16 ulp of the final add's operands
    t = (n * (1.0 + scale.index_select(0, idx))).float().abs() + shift.index_select(0, idx).float().abs()
    assert (np.abs(O.bf16_to_f32(got) - ref.float().numpy()) <= t.numpy() * 2.0**-5).all()


def test_epilogue_silu_takes_bf16_cuda_tensors_only():
    with pytest.raises(ValueError, match="bf16 CUDA"):
        ffn.silu_bf16(torch.zeros(4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="bf16 CUDA"):
        ffn.silu_bf16(torch.zeros(4))
