"""The reference's own B200 path beside this library's kernels, on the same seeded inputs.

The reference runs its Triton rotate+quantise kernels (rotate_quant_factored_kernel, the pipeline's default, and
rotate_quant_kernel; int8.py:194-262) and, on sm_100, torch._int_mm (cuBLASLt) plus its Triton rescale kernel for
the GEMM (int8.py:353-364, 315-324).  Its module is loaded by file path from its installed copy (baseline/_ref);
these tests skip when that copy or Triton is missing.

* int32 accumulator and dequantised output: bitwise equal to torch._int_mm and to the reference's int8_matmul on the
  same codes (both use the exact int32 sum and the ``(acc * sa) * sb`` multiply order).
* codes and scales: the reference's Triton kernels accumulate the rotation on tensor cores in fp32, while this
  library (and the oracle) rounds the exact sum once.  They are held to the reference's own bound between its two
  kernels (tests/test_int8.py:113-116): at most 1e-5 of the codes differ, by at most one, and scales within rtol
  1e-5.  The fraction that is bit-identical is reported.
"""

from __future__ import annotations

import pytest
import torch

import bench
from hyperflow_h3_flash_b200 import _lib
from hyperflow_h3_flash_b200 import int8 as I
from hyperflow_h3_flash_b200 import synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"
G = 256


@pytest.fixture(scope="module")
def ref():
    mod, why = bench.load_reference_int8()
    if mod is None:
        pytest.skip(why)
    try:
        kernels = mod._kernels()
    except Exception as e:  # noqa: BLE001 - a broken Triton install is a reason to skip, reported
        pytest.skip(f"the reference's _kernels() failed: {e}")
    if kernels is None:
        pytest.skip("Triton is not importable: the reference has no CUDA kernels")
    yield mod, kernels
    mod.set_kernel_options(rotate_quant="dense", int8_gemm="auto")


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.lib().convrot_poll_error(None) == 0


def inputs(M: int, K: int, seed: int) -> torch.Tensor:
    x = synthetic.activations(M, K, seed=seed)
    x[1] = 0  # an all-zero row: the 1e-12 floor of the scale
    x[2, :G] = 0  # an all-zero group
    x[3::7, ::97] *= 30  # the reference's own outlier pattern (tests/test_int8.py:101), on every 7th row
    return x.to(DEV)


@pytest.mark.parametrize("M,N,K", [(300, 256, 14336), (4096, 5120, 5120), (333, 5120, 4096), (32768, 5120, 5120)])
def test_int32_accumulator_and_output_are_bitwise_the_references(ref, M, N, K):
    mod, kernels = ref
    gen = torch.Generator().manual_seed(M + N + K)
    q = torch.randint(-127, 128, (M, K), generator=gen, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (N, K), generator=gen, dtype=torch.int8).to(DEV)
    sa = (torch.rand(M, generator=gen) * 1e-2 + 1e-4).to(DEV)
    sb = (torch.rand(N, generator=gen) * 1e-3 + 1e-5).to(DEV)
    assert torch.equal(I.int8_mm_acc(q, w), torch._int_mm(q, w.t()))
    mod.set_kernel_options(int8_gemm="cublas")
    assert torch.equal(I.int8_matmul(q, w, sa, sb), kernels.int8_matmul(q, w, sa, sb))


@pytest.mark.parametrize("option", ["factored", "dense"])
@pytest.mark.parametrize("M,K", [(4096, 5120), (333, 13824)])
def test_codes_and_scales_within_the_references_own_bound(ref, option, M, K):
    mod, kernels = ref
    x = inputs(M, K, seed=K)
    mod.set_kernel_options(rotate_quant=option)
    qr, sr = kernels.rotate_quant(x, G)
    q, s = I.rotate_quant(x, G)
    diff = (qr.to(torch.int16) - q.to(torch.int16)).abs()
    frac = float((diff != 0).double().mean())
    print(f"{option} M={M} K={K}: codes differing {frac:.3g} (max |d| {int(diff.max())}), "
          f"scales bit-identical {float((s == sr).double().mean()):.6f}")
    assert frac <= 1e-5 and int(diff.max()) <= 1
    torch.testing.assert_close(s, sr, rtol=1e-5, atol=0)


def test_layer_forward_is_bitwise_the_references_where_codes_agree(ref):
    """The reference's Int8RotLinear.forward on CUDA (its kernels) against this library's module, same weights:
    rows whose codes and scale agree give bitwise the same output (the GEMM and epilogue are bitwise equal)."""
    mod, kernels = ref
    M, K, N = 2048, 5120, 1024
    w = synthetic.linear_weights(K, N, bias=False, group=G, seed_offset=3)
    theirs = mod.Int8RotLinear(K, N, G)
    theirs.qweight.data.copy_(w.qweight)
    theirs.wscale.data.copy_(w.wscale)
    ours = I.Int8RotLinear(K, N, G)
    synthetic.load_into(ours, w)
    theirs, ours = theirs.to(DEV), ours.to(DEV)
    x = inputs(M, K, seed=11)
    mod.set_kernel_options(rotate_quant="factored", int8_gemm="auto")
    y_ref, y = theirs(x), ours(x)
    qr, sr = kernels.rotate_quant(x, G)
    q, s = I.rotate_quant(x, G)
    same = ((qr == q).all(dim=1) & (sr == s)).to(DEV)
    # about one row in eight has a scale a few ulp apart (its division and tensor-core sums, see below)
    assert same.float().mean() >= 0.75
    assert torch.equal(y_ref[same], y[same])


def test_triton_division_mode_is_closer_to_the_reference_kernels(ref):
    """The reference's Triton `/` is not IEEE division.  Mode CONVROT_ROUND_TRITON divides with div.full.f32 and
    lands nearer the reference's kernels than the exact mode: fewer differing codes and scales, every difference still
    within the reference's own bound.  What differs after that comes from the reference's tensor-core fp32 sums of
    the rotation (its dense and factored kernels also differ from each other)."""
    mod, kernels = ref
    x = inputs(8192, 5120, seed=5)
    counts = {}
    for option in ("factored", "dense"):
        mod.set_kernel_options(rotate_quant=option)
        qr, sr = kernels.rotate_quant(x, G)
        for mode in (_lib.ROUND_KERNEL, _lib.ROUND_TRITON):
            q, s = I.rotate_quant(x, G, rounding=mode)
            d = (qr.to(torch.int16) - q.to(torch.int16)).abs()
            counts[option, mode] = (int((d != 0).sum()), int((s != sr).sum()))
            assert int(d.max()) <= 1 and float((d != 0).double().mean()) <= 1e-5
            torch.testing.assert_close(s, sr, rtol=1e-5, atol=0)
    for option in ("factored", "dense"):
        assert counts[option, _lib.ROUND_TRITON][0] <= counts[option, _lib.ROUND_KERNEL][0], counts
        assert counts[option, _lib.ROUND_TRITON][1] <= counts[option, _lib.ROUND_KERNEL][1], counts
    mod.set_kernel_options(rotate_quant="factored")
    q_f, s_f = kernels.rotate_quant(x, G)
    mod.set_kernel_options(rotate_quant="dense")
    q_d, s_d = kernels.rotate_quant(x, G)
    between = int((q_f != q_d).sum())
    print(f"codes / scales differing from the reference (factored, dense) x (exact, div.full): {counts}; "
          f"the reference's two kernels differ from each other in {between} codes")
