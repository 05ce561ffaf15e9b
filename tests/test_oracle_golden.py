"""The CPU oracle against golden vectors produced by the reference itself (tests/golden/make_golden.py).

These pin the oracle before anything is checked against it: the Hadamard rotation, the checkpoint recipe, the
reference's Triton rotate+quantise kernels (int8.py:194-262), its GEMM and rescale epilogues (int8.py:283-324) and
its CPU path ``_forward_torch`` (int8.py:173-179).
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import GOLDEN


def load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("group", [4, 16, 64, 256])
def test_regular_hadamard_matches_reference(group):
    h = O.regular_hadamard(group)
    assert np.array_equal(h.astype(np.float32), load("hadamard.npz")[f"h{group}"])
    np.testing.assert_allclose(h @ h.T, np.eye(group), atol=1e-12)  # orthonormal (test_int8.py:39-43)
    assert np.array_equal(h, h.T)


def test_hadamard_rejects_and_factors_match_reference():
    g = load("hadamard.npz")
    for size in g["rejected"]:
        with pytest.raises(ValueError):
            O.regular_hadamard(int(size))
    for size, (ga, gb) in zip(g["factor_groups"], g["factors"]):
        expect = None if ga == 0 else (int(ga), int(gb))
        assert O.hadamard_factors(int(size)) == expect
        if expect:
            assert np.array_equal(np.kron(O.regular_hadamard(ga), O.regular_hadamard(gb)),
                                  O.regular_hadamard(int(size)))


@pytest.mark.parametrize("group", [16, 64, 256])
def test_rotate_quant_is_bitwise_the_reference_kernel_with_an_exact_dot(group):
    t = load("triton_kernels.npz")
    q, s = O.rotate_quant(t["x"], group)
    assert np.array_equal(q, t[f"dense_exact_g{group}_q"])
    assert np.array_equal(s, t[f"dense_exact_g{group}_s"])


@pytest.mark.parametrize("kernel", ["dense_fp32_g16", "dense_fp32_g64", "dense_fp32_g256", "factored_exact_g256",
                                    "factored_fp32_g256"])
def test_rotate_quant_within_the_reference_tolerance_of_inexact_dots(kernel):
    # The reference's own bound between two rotations (tests/test_int8.py:113-116).
    t = load("triton_kernels.npz")
    q, s = O.rotate_quant(t["x"], int(kernel.rsplit("g", 1)[1]))
    gq, gs = t[f"{kernel}_q"], t[f"{kernel}_s"]
    np.testing.assert_allclose(s, gs, rtol=1e-5, atol=0)
    assert (q != gq).mean() <= 1e-5
    assert np.abs(q.astype(np.int32) - gq).max() <= 1


def test_gemm_and_rescale_epilogues_are_bitwise_the_reference():
    t = load("triton_kernels.npz")
    acc = O.int8_gemm(t["gemm_a"], t["gemm_b"])
    assert np.array_equal(acc, t["rescale_acc"])
    out = O.epilogue(acc, t["gemm_sa"], t["gemm_sb"])
    assert np.array_equal(out, t["gemm_out"])
    assert np.array_equal(out, t["rescale_out"])


def test_checkpoint_recipe_matches_reference():
    c = load("cpu_forward.npz")
    for case, group in (("a", 16), ("c", 256)):
        qw, ws = O.quantize_weight(c[f"{case}_weight"], group)
        assert np.array_equal(qw, c[f"{case}_qweight"])
        assert np.array_equal(ws, c[f"{case}_wscale"])


def test_cpu_path_restatement_is_bitwise_the_reference_forward_torch():
    c = load("cpu_forward.npz")
    q, s = O.rotate_quant_cpu(c["b_x"], 256)
    y = O.epilogue(O.int8_gemm(q, c["b_qweight"]), s, c["b_wscale"])
    assert np.array_equal(y, c["b_y"])
    assert np.array_equal(O.forward_cpu_port(c["b_x"], c["b_qweight"], c["b_wscale"], 256), c["b_y"])
    # fp32 input, group 16: the module casts to bf16 first (int8.py:163).
    x = O.f32_to_bf16(c["a_x"].reshape(-1, 128))
    q, s = O.rotate_quant_cpu(x, 16)
    y = O.bf16_to_f32(O.epilogue(O.int8_gemm(q, c["a_qweight"]), s, c["a_wscale"]))
    assert np.array_equal(y, c["a_y"].reshape(-1, 96))


def test_exact_rotation_survives_wide_exponent_spans():
    # A group holding 2^100 and 2^-120 needs the 320-bit path; the result must equal the exact sum rounded once.
    x = np.zeros((1, 16), np.float32)
    x[0, 0] = 2.0**100
    x[0, 1] = 2.0**-120
    x[0, 2] = 1.5
    bits = O.f32_to_bf16(x)
    y, yb, slow = O.rotate(bits, 16)
    assert slow == 1
    h = O.regular_hadamard(16)
    # exact: 2^100*h0j + 2^-120*h1j + 1.5*h2j with |h|=1/4; the tiny terms vanish after rounding to fp32.
    expect = (x.astype(np.float64) @ h).astype(np.float32)
    assert np.array_equal(y, expect)


def test_rounding_is_half_to_even_at_ties():
    # Rows whose rotated values land exactly on .5 codes: x = e0 * c gives y_j = c/4 * sign (group 16).
    x = np.zeros((1, 16), np.float32)
    x[0, 0] = 254.0  # amax = 63.5 -> scale = 0.5 exactly; every y = +-63.5 -> y*inv = +-127 exactly
    x2 = x.copy()
    x2[0, 0], x2[0, 1] = 254.0, 2.0  # y in {+-64, +-63}: codes 127*64/64 ... checked against float math below
    for row in (x, x2):
        q, s = O.rotate_quant(O.f32_to_bf16(row), 16)
        y = (row.astype(np.float64) @ O.regular_hadamard(16)).astype(np.float32)
        amax = np.float32(np.abs(y).max())
        scale = np.float32(np.float64(max(amax, np.float32(1e-12))) / 127.0)
        inv = np.float32(1.0 / np.float64(scale))
        expect = np.clip(np.rint((y * inv).astype(np.float32)), -127, 127).astype(np.int8)
        assert s[0] == scale and np.array_equal(q, expect)
