"""Host-side API of the drop-in module, mirroring the reference's own tests (tests/test_int8.py) on the CPU."""

from __future__ import annotations

import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from hyperflow_h3_flash_b200 import int8 as I
from hyperflow_h3_flash_b200 import synthetic
from oracle import oracle as O
from tests.conftest import GOLDEN


@pytest.mark.parametrize("group", [4, 16, 64, 256])
def test_regular_hadamard_is_the_reference_matrix(group):
    h = I.regular_hadamard(group)
    golden = np.load(os.path.join(GOLDEN, "hadamard.npz"))[f"h{group}"]
    assert np.array_equal(h.numpy(), golden)
    torch.testing.assert_close(h.double() @ h.double().T, torch.eye(group, dtype=torch.float64))


def test_regular_hadamard_rejects_non_powers_of_four():
    for group in (32, 128):
        with pytest.raises(ValueError):
            I.regular_hadamard(group)


@pytest.mark.parametrize("group", [256, 1024, 4096])
def test_hadamard_factors_rebuild_the_rotation(group):
    ga, gb = I.hadamard_factors(group)
    assert ga >= 16 and gb >= 16
    torch.testing.assert_close(torch.kron(I.regular_hadamard(ga), I.regular_hadamard(gb)), I.regular_hadamard(group))
    assert I.hadamard_factors(16) is None and I.hadamard_factors(64) is None


def test_kernel_options_are_checked():
    saved = dict(I.KERNEL_OPTIONS)
    try:
        assert I.KERNEL_OPTIONS == {"int8_gemm": "auto", "rotate_quant": "dense"}
        with pytest.raises(ValueError, match="int8_gemm"):
            I.set_kernel_options(int8_gemm="cutlass")
        with pytest.raises(ValueError, match="rotate_quant"):
            I.set_kernel_options(rotate_quant="fast")
        I.set_kernel_options(int8_gemm="triton", rotate_quant="factored")
        assert I.resolve_int8_gemm(torch.device("cpu")) == "tcgen05"
    finally:
        I.KERNEL_OPTIONS.update(saved)


def test_state_is_two_frozen_parameters_and_extensions_are_opt_in():
    layer = I.Int8RotLinear(64, 32, group=16)
    assert set(layer.state_dict()) == {"qweight", "wscale"}
    assert not list(layer.buffers())
    assert not any(p.requires_grad for p in layer.parameters())
    full = I.Int8RotLinear(64, 32, group=16, bias=True, rank=8)
    assert set(full.state_dict()) == {"qweight", "wscale", "bias", "down.weight", "up.weight"}
    assert full.down.weight.shape == (8, 64) and full.up.weight.shape == (32, 8)
    assert not any(p.requires_grad for p in full.parameters())
    with pytest.raises(ValueError):
        I.Int8RotLinear(100, 32, group=16)


def test_cpu_forward_is_bitwise_the_reference_torch_path():
    c = np.load(os.path.join(GOLDEN, "cpu_forward.npz"))
    layer = I.Int8RotLinear(1024, 256, group=256)
    layer.qweight.copy_(torch.from_numpy(c["b_qweight"]))
    layer.wscale.copy_(torch.from_numpy(c["b_wscale"]))
    x = torch.from_numpy(c["b_x"].view(np.int16)).view(torch.bfloat16)
    y = layer(x)
    assert np.array_equal(y.view(torch.int16).numpy().view(np.uint16), c["b_y"])
    layer = I.Int8RotLinear(128, 96, group=16)
    layer.qweight.copy_(torch.from_numpy(c["a_qweight"]))
    layer.wscale.copy_(torch.from_numpy(c["a_wscale"]))
    y = layer(torch.from_numpy(c["a_x"]))
    assert y.dtype == torch.float32 and y.shape == (5, 7, 96)
    assert np.array_equal(y.numpy(), c["a_y"])


def test_int8_linear_matches_dense():
    # tests/test_int8.py:51-63 on this module
    torch.manual_seed(0)
    weight = torch.randn(96, 128) * 0.05
    x = torch.randn(5, 7, 128)
    layer = I.Int8RotLinear(128, 96, group=16)
    qw, ws = synthetic.quantize_weight(weight, 16)
    layer.qweight.copy_(qw)
    layer.wscale.copy_(ws)
    y = layer(x)
    reference = x @ weight.T
    assert y.shape == (5, 7, 96) and y.dtype == x.dtype
    assert (y.float() - reference).norm() / reference.norm() < 0.02


def test_synthetic_checkpoint_recipe_matches_the_reference():
    c = np.load(os.path.join(GOLDEN, "cpu_forward.npz"))
    for case, group in (("a", 16), ("c", 256)):
        qw, ws = synthetic.quantize_weight(torch.from_numpy(c[f"{case}_weight"]), group)
        assert np.array_equal(qw.numpy(), c[f"{case}_qweight"])
        assert np.array_equal(ws.numpy(), c[f"{case}_wscale"])


def test_cpu_forward_with_bias_and_low_rank_is_the_composite():
    M, K, N, r = 9, 256, 64, 16
    x = synthetic.activations(M, K)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=16)
    layer = I.Int8RotLinear(K, N, group=16, bias=True, rank=r)
    synthetic.load_into(layer, w)
    plain = I.Int8RotLinear(K, N, group=16)
    plain.qweight.copy_(w.qweight)
    plain.wscale.copy_(w.wscale)
    expect = plain(x) + w.bias + (x @ w.down.t()) @ w.up.t()
    assert torch.equal(layer(x), expect)


def test_shared_quantization_works_under_inference_mode():
    # tests/test_int8.py:176-185
    calls = []
    kernels = SimpleNamespace(rotate_quant=lambda x2, group: calls.append(1) or (x2, group))
    to_q, to_k = I.Int8RotLinear(16, 16, group=16), I.Int8RotLinear(16, 16, group=16)
    to_q.keep_input = True
    with torch.inference_mode():
        x = torch.randn(4, 16)
        to_q._quantize(x, x, kernels)
        to_k._quantize(x, x, kernels)
    assert len(calls) == 1 and not I.Int8RotLinear._last_input


def test_oracle_semantics_differ_from_cpu_path_only_by_the_rotation_rounding():
    # The kernel path (fp32 rotation, multiply by 1/s) and the torch path (bf16 rotation, divide by s) give nearby
    # codes: the reference accepts both for the same layer.
    x = synthetic.activations(64, 1024)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    qk, sk = O.rotate_quant(xb, 256)
    qc, sc = O.rotate_quant_cpu(xb, 256)
    assert np.abs(qk.astype(int) - qc).max() <= 1
    np.testing.assert_allclose(sk, sc, rtol=1e-2)


def test_gated_residual_on_cpu_is_the_bf16_composition():
    import torch

    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic

    w = synthetic.linear_weights(512, 256, rank=16, bias=True, group=256)
    layer = I.Int8RotLinear(512, 256, 256, bias=True, rank=16)
    synthetic.load_into(layer, w)
    x = synthetic.activations(20, 512, seed=3)
    res = synthetic.activations(20, 256, seed=4)
    gate = (torch.randn(3, 256) * 0.1).to(torch.bfloat16)
    idx = torch.arange(20) % 3
    y = layer(x)
    assert torch.equal(layer(x, residual=res, gate=gate, gate_index=idx), res + gate.index_select(0, idx) * y)
    assert torch.equal(layer(x, residual=res, gate=gate[1]), res + gate[1] * y)
    assert torch.equal(layer(x, residual=res), res + y)


def test_save_and_load_keep_storage_dtypes_and_outputs(tmp_path):
    """tests/test_transformer.py:164-175 on this layer: a saved state dict reloads with int8 / fp32 / bf16 storage
    and the same outputs."""
    import torch

    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic

    w = synthetic.linear_weights(256, 128, rank=16, bias=True, group=64)
    layer = I.Int8RotLinear(256, 128, 64, bias=True, rank=16)
    synthetic.load_into(layer, w)
    path = tmp_path / "layer.pt"
    torch.save(layer.state_dict(), path)
    fresh = I.Int8RotLinear(256, 128, 64, bias=True, rank=16)
    fresh.load_state_dict(torch.load(path))
    dtypes = {k: v.dtype for k, v in fresh.state_dict().items()}
    assert dtypes == {"qweight": torch.int8, "wscale": torch.float32, "bias": torch.bfloat16,
                      "down.weight": torch.bfloat16, "up.weight": torch.bfloat16}
    x = synthetic.activations(20, 256, seed=5)
    assert torch.equal(fresh(x), layer(x))
