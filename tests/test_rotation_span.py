"""Facts about the rotation that the G = 256 kernel relies on (CPU): exponent spans of 256-groups in the bench's
synthetic activations, and the exactness of the kernel's per-team row order.

The rotation kernels sum each group in fp64 on integer-form values. That sum is exact while a group's nonzero
magnitudes span at most 37 binades: floor(log2 max|x|) - floor(log2 min|x|) <= 37 for G = 256. This test pins that
every group of the bench's inputs lies inside that domain, so the bitwise parity the GPU tests check also holds
for the timed data.

It also records how often a narrower exact form would have to fall back:
- an int32 fixed-point sum (8 significand bits, 8 bits of growth over 256 terms and the sign leave 14 binades);
- a two-limb fp32 sum (25 binades).
With the inputs' 1 % outlier channels at 20x, about one group in six exceeds the int32 width, and so do about half
of the warps that each rotate four groups.
"""

from __future__ import annotations

import numpy as np

from hyperflow_h3_flash_b200 import synthetic


def spans(M: int, K: int, outlier_scale: float) -> np.ndarray:
    x = np.abs(synthetic.activations(M, K, seed=1, outlier_scale=outlier_scale).float().numpy())
    g = x.reshape(M, K // 256, 256)
    mx = g.max(-1)
    mn = np.where(g > 0, g, np.inf).min(-1)
    return np.floor(np.log2(mx)) - np.floor(np.log2(mn))


def test_bench_inputs_lie_inside_the_exact_domain_of_the_fp64_rotation():
    s = spans(2048, 5120, 20.0)
    assert s.max() <= 37
    int32_groups = float((s > 14).mean())
    int32_warps = float((s > 14).reshape(2048, 5, 4).any(-1).mean())
    two_limb = float((s > 25).mean())
    print(f"groups beyond int32's 14 binades: {int32_groups:.3f} (warps of four groups: {int32_warps:.3f}); "
          f"beyond two fp32 limbs' 25: {two_limb:.4f}")
    assert 0.1 < int32_groups < 0.25 and int32_warps > 0.4
    assert two_limb < 0.01


def test_without_outlier_channels_few_groups_exceed_the_int32_width():
    s = spans(2048, 5120, 1.0)
    assert s.max() <= 37
    assert float((s > 14).mean()) < 0.05


def test_row_order_a_xor_j_permutes_the_column_transform_exactly():
    """The G = 256 kernel's team j loads row a ^ j of its 16 x 16 group matrix into register a (j = 0..3) so that
    the four teams of a warp read different banks.  That is exact because H4' (the integer H4, -1 where
    row ^ column == 3) satisfies H4'[i ^ j][k] = H4'[i][k ^ j]: the 16-point transform kron(H4', H4') of the
    row-permuted input is the transform's output permuted the same way, for any input (checked here on random
    integers, where every sum is exact)."""
    from oracle import oracle as O

    h16 = O.regular_hadamard(16) * 4  # kron(H4', H4') with integer entries
    h4 = O.regular_hadamard(4) * 2
    idx = np.arange(4)
    for j in range(4):
        assert np.array_equal(h4[idx ^ j], h4[:, idx ^ j])
    rng = np.random.default_rng(3)
    x = rng.integers(-(2**20), 2**20, size=(64, 16)).astype(np.float64)
    a = np.arange(16)
    for j in range(4):
        permuted_in = x[:, a ^ j] @ h16  # register a holds row a ^ j
        assert np.array_equal(permuted_in, (x @ h16)[:, a ^ j])  # register k holds output row k ^ j
