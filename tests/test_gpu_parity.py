"""Parity of the sm_100a kernels with the CPU oracle (and with the reference's own kernels' golden outputs).

Bit-exact: int8 codes, per-token scales, int32 accumulators, and the bias-free bf16 output (the reference's
``(acc * sa) * sb`` epilogue, int8.py:311, 324). Within tolerance (no reference counterpart): the fused bias and
low-rank output, max |err| / max |ref| <= 1e-2 and cosine >= 0.9999 against the composite reference
``int8 + bias + up(down(x))``, and the low-rank ``x . down^T`` within one bf16 rounding plus the fp32
accumulation bound.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from hyperflow_h3_flash_b200 import _lib
from hyperflow_h3_flash_b200 import int8 as I
from hyperflow_h3_flash_b200 import synthetic
from oracle import oracle as O
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

DEV = "cuda"


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def edge_rows(x: torch.Tensor, group: int) -> torch.Tensor:
    x = x.clone()
    if x.shape[0] > 3:
        x[1] = 0  # all-zero row: the 1e-12 floor of the scale
        x[2, :group] = 0  # an all-zero group
        x[3, 5] = 3.0e4  # a large outlier (amax far above the rest)
    return x


def close(out: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    out = out.astype(np.float64)
    ref = ref.astype(np.float64)
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    cos = (out * ref).sum() / np.sqrt((out * out).sum() * (ref * ref).sum())
    return float(err), float(cos)


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.lib().convrot_poll_error(None) == 0


@pytest.fixture(params=[2, 1], ids=["rot2col", "rot1col"])
def rotate_variant(request):
    """Group-256 rotation on the two-column team kernel and on the one-column kernel."""
    _lib.check(_lib.lib().convrot_set_rotate_variant(request.param), "convrot_set_rotate_variant")
    yield request.param
    _lib.lib().convrot_set_rotate_variant(0)


@pytest.fixture(params=[1, 2], ids=["gemm1sm", "gemm2sm"])
def gemm_mode(request):
    """Runs a test on the 1-SM (128x256 tiles) and on the 2-SM (cta_group::2, 256x256 per CTA pair) kernel."""
    _lib.check(_lib.lib().convrot_set_gemm_mode(request.param), "convrot_set_gemm_mode")
    yield request.param
    _lib.lib().convrot_set_gemm_mode(0)


# ---------------------------------------------------------------------------------------------- rotate + quantise


@pytest.mark.parametrize("M,K,group", [
    (1, 256, 256), (17, 1024, 256), (70, 1024, 256), (333, 4096, 256), (64, 5120, 256), (40, 13824, 256),
    (33, 512, 16), (33, 1024, 64), (33, 64, 4), (5, 16384, 256), (3, 32768, 256), (129, 2048, 16),
    # more rows than CTAs: each CTA cycles its row ring several times (a one-buffer ring at K = 13824)
    (4000, 13824, 256), (4000, 13824, 16), (2500, 16384, 256), (5000, 5120, 256),
])
def test_rotate_quant_is_bitwise_the_oracle(M, K, group, rotate_variant):
    x = edge_rows(synthetic.activations(M, K, seed=M + K), group)
    q, s = I.rotate_quant(x.to(DEV), group)
    q_ref, s_ref = O.rotate_quant(bits(x), group)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("group", [16, 64, 256])
def test_rotate_quant_is_bitwise_the_reference_kernel(group, rotate_variant):
    t = np.load(os.path.join(GOLDEN, "triton_kernels.npz"))
    q, s = I.rotate_quant(from_bits(t["x"]).to(DEV), group)
    assert np.array_equal(q.cpu().numpy(), t[f"dense_exact_g{group}_q"])
    assert np.array_equal(s.cpu().numpy(), t[f"dense_exact_g{group}_s"])
    # and within the reference's own tolerance of its inexact-dot runs (tests/test_int8.py:113-116)
    gq, gs = t[f"dense_fp32_g{group}_q"], t[f"dense_fp32_g{group}_s"]
    np.testing.assert_allclose(s.cpu().numpy(), gs, rtol=1e-5, atol=0)
    assert (q.cpu().numpy() != gq).mean() <= 1e-5


@pytest.mark.parametrize("M,K,group", [(8, 1024, 256), (16, 512, 16), (3, 256, 64), (1, 5120, 256)])
def test_torch_rounding_mode_is_bitwise_the_reference_cpu_path(M, K, group, rotate_variant):
    x = synthetic.activations(M, K, seed=11)
    q, s = I.rotate_quant_torch_rounding(x.to(DEV), group)
    q_ref, s_ref = O.rotate_quant_cpu(bits(x), group)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


# ---------------------------------------------------------------------------------------------- GEMM


def codes(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)


@pytest.mark.parametrize("M,N,K", [
    (1, 256, 256), (17, 96, 512), (129, 300, 640), (300, 256, 14336), (256, 512, 5120), (333, 5120, 4096),
    (200, 1000, 128), (128, 256, 16),
])
def test_int32_accumulator_is_bitwise_the_oracle(M, N, K, gemm_mode):
    a, b = codes(M, K, 1), codes(N, K, 2)
    acc = I.int8_mm_acc(a.to(DEV), b.to(DEV))
    assert np.array_equal(acc.cpu().numpy(), O.int8_gemm(a.numpy(), b.numpy()))


@pytest.mark.parametrize("M,N,K", [(17, 96, 512), (129, 300, 640), (300, 256, 14336), (333, 5120, 4096)])
def test_bf16_epilogue_is_bitwise_the_oracle(M, N, K, gemm_mode):
    a, b = codes(M, K, 3), codes(N, K, 4)
    g = torch.Generator().manual_seed(5)
    sa = torch.rand(M, generator=g) * 0.05 + 1e-4
    sb = torch.rand(N, generator=g) * 1e-3 + 1e-6
    y = I.int8_matmul(a.to(DEV), b.to(DEV), sa.to(DEV), sb.to(DEV))
    ref = O.epilogue(O.int8_gemm(a.numpy(), b.numpy()), sa.numpy(), sb.numpy())
    assert np.array_equal(bits(y), ref)


def test_gemm_and_rescale_are_bitwise_the_reference_kernels(gemm_mode):
    t = np.load(os.path.join(GOLDEN, "triton_kernels.npz"))
    dev = lambda k: torch.from_numpy(t[k]).to(DEV)  # noqa: E731
    y = I.int8_matmul(dev("gemm_a"), dev("gemm_b"), dev("gemm_sa"), dev("gemm_sb"))
    assert np.array_equal(bits(y), t["gemm_out"])
    acc = I.int8_mm_acc(dev("gemm_a"), dev("gemm_b"))
    assert np.array_equal(acc.cpu().numpy(), t["rescale_acc"])


# ---------------------------------------------------------------------------------------------- low-rank + bias


# M <= 1024 splits K over a cluster of CTAs (2-8 by K); 1025 rows and up run unsplit
@pytest.mark.parametrize("M,K,r", [(40, 1024, 16), (333, 4096, 32), (256, 5120, 64), (17, 520, 48),
                                   (1024, 4096, 256), (1025, 1024, 96), (17, 256, 16), (5, 8192, 128)])
def test_lowrank_down_within_one_bf16_ulp(M, K, r):
    x = synthetic.activations(M, K, seed=7)
    g = torch.Generator().manual_seed(9)
    down = (torch.randn(r, K, generator=g) * 0.01).to(torch.bfloat16)
    xa = I.lowrank_down(x.to(DEV), down.to(DEV))
    ref = O.bf16_to_f32(O.lowrank_down(bits(x), bits(down.t().contiguous())))
    out = xa.float().cpu().numpy()
    # one bf16 rounding of the result plus the fp32 accumulation bound K * 2^-24 * (|x| . |A|)
    mag = np.abs(O.bf16_to_f32(bits(x))).astype(np.float64) @ np.abs(O.bf16_to_f32(bits(down.t().contiguous())))
    bound = np.abs(ref) * 2.0**-7 + K * 2.0**-24 * mag
    assert (np.abs(out - ref) <= bound).all()
    assert (out == ref).mean() > 0.95  # almost every value is the correctly rounded one


@pytest.mark.parametrize("M,K,N,r,group", [
    (40, 1024, 256, 16, 256), (333, 4096, 5120, 32, 256), (256, 4096, 5120, 32, 256), (256, 5120, 512, 64, 256),
    (17, 512, 300, 48, 16), (130, 2048, 1000, 0, 64),
    (300, 1024, 512, 128, 256), (129, 2048, 768, 192, 256), (520, 512, 256, 256, 256), (77, 1024, 320, 80, 256),
])  # (256 | 333, 4096 -> 5120, r = 32): config 5; r > 64 streams the rank through the epilogue in chunks of 64
def test_fused_bias_and_low_rank_within_tolerance(M, K, N, r, group, gemm_mode):
    x = synthetic.activations(M, K, seed=13)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=group)
    q, s = I.rotate_quant(x.to(DEV), group)
    xa = I.lowrank_down(x.to(DEV), w.down.to(DEV)) if r else None
    y = I.convrot_matmul(q, w.qweight.to(DEV), s, w.wscale.to(DEV), bias=w.bias.to(DEV), xa=xa,
                         up=w.up.to(DEV) if r else None)
    A = bits(w.down.t().contiguous()) if r else None
    B = bits(w.up.t().contiguous()) if r else None
    # against the oracle's fused epilogue (same fp32 formula) ...
    o = O.convrot_linear(bits(x), w.qweight.numpy(), w.wscale.numpy(), group, bits(w.bias), A, B)
    out = y.float().cpu().numpy()
    err, cos = close(out, O.bf16_to_f32(o["out"]))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    # ... and against the composite of the reference's modules
    ref = O.bf16_to_f32(O.composite_reference(bits(x), w.qweight.numpy(), w.wscale.numpy(), group, bits(w.bias), A, B))
    err, cos = close(out, ref)
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    # every value is within a couple of bf16 ulps of the oracle's fused value
    o32 = O.bf16_to_f32(o["out"])
    assert (np.abs(out - o32) <= np.abs(o32) * 2.0**-6 + 1e-3 * np.abs(o32).max()).all()


# ---------------------------------------------------------------------------------------------- the layer


@pytest.mark.parametrize("M", [8, 16, 17, 333])
def test_layer_forward_matches_the_reference_regime(M):
    K, N, G = 1024, 512, 256
    x = synthetic.activations(M, K, seed=21)
    w = synthetic.linear_weights(K, N, bias=False, group=G)
    layer = I.Int8RotLinear(K, N, G)
    synthetic.load_into(layer, w)
    y = layer.to(DEV)(x.to(DEV))
    if M >= I._MIN_KERNEL_ROWS:
        q, s = O.rotate_quant(bits(x), G)  # the reference's CUDA-kernel arithmetic
    else:
        q, s = O.rotate_quant_cpu(bits(x), G)  # its torch path, used below 17 rows (int8.py:164-167)
    ref = O.epilogue(O.int8_gemm(q, w.qweight.numpy()), s, w.wscale.numpy())
    assert np.array_equal(bits(y), ref)


def test_layer_with_bias_and_low_rank_matches_the_composite():
    M, K, N, r, G = 257, 5120, 640, 32, 256
    x = synthetic.activations(M, K, seed=3)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=G)
    layer = I.Int8RotLinear(K, N, G, bias=True, rank=r)
    synthetic.load_into(layer, w)
    y = layer.to(DEV)(x.to(DEV).reshape(1, M, K))
    assert y.shape == (1, M, N)
    ref = O.bf16_to_f32(O.composite_reference(bits(x), w.qweight.numpy(), w.wscale.numpy(), G, bits(w.bias),
                                              bits(w.down.t().contiguous()), bits(w.up.t().contiguous())))
    err, cos = close(y.float().cpu().numpy().reshape(M, N), ref)
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_q_k_v_share_one_quantization(monkeypatch):
    # tests/test_int8.py:149-173 on this module's kernels
    kernels = I._kernels()
    calls = []
    rotate_quant = kernels.rotate_quant
    monkeypatch.setattr(kernels, "rotate_quant", lambda *a: calls.append(1) or rotate_quant(*a))

    def layer(seed):
        w = synthetic.linear_weights(1024, 512, bias=False, group=256, seed_offset=seed)
        m = I.Int8RotLinear(1024, 512, 256)
        synthetic.load_into(m, w)
        return m.to(DEV)

    to_q, to_k, to_v = layer(0), layer(1), layer(2)
    x = synthetic.activations(1000, 1024).to(DEV)
    to_q.keep_input = to_k.keep_input = True
    shared = [to_q(x), to_k(x), to_v(x)]
    assert len(calls) == 1 and not I.Int8RotLinear._last_input
    to_q.keep_input = to_k.keep_input = False
    separate = [to_q(x), to_k(x), to_v(x)]
    assert len(calls) == 4
    for a, b in zip(shared, separate, strict=True):
        assert torch.equal(a, b)
    to_q.keep_input = True
    to_q(x)
    x.mul_(2)
    to_k(x)
    to_q(x)
    to_k(x.clone())
    assert len(calls) == 8


# ---------------------------------------------------------------------------------------------- full-size shapes


@pytest.mark.parametrize("M,K,N", [(32768, 5120, 5120), (32761, 5120, 5120)])
def test_full_size_sampled_rows_are_bitwise_the_oracle(M, K, N, gemm_mode):
    """Configs 2 and 5 (M = 32761: a ragged tail): every output row is computed, sampled rows checked bit-exact."""
    G = 256
    x = synthetic.activations(M, K, seed=0)
    w = synthetic.linear_weights(K, N, bias=False, group=G)
    xd = x.to(DEV)
    q, s = I.rotate_quant(xd, G)
    y = I.int8_matmul(q, w.qweight.to(DEV), s, w.wscale.to(DEV))
    rows = np.unique(np.concatenate([np.arange(4), np.arange(M - 4, M),
                                     np.random.default_rng(0).integers(0, M, 24)]))
    q_ref, s_ref = O.rotate_quant(bits(x[rows]), G)
    assert np.array_equal(q[rows].cpu().numpy(), q_ref)
    assert np.array_equal(s[rows].cpu().numpy(), s_ref)
    ref = O.epilogue(O.int8_gemm(q_ref, w.qweight.numpy()), s_ref, w.wscale.numpy())
    assert np.array_equal(bits(y[rows]), ref)
    # size-independent check over all rows: the output's row norms are finite and the zero-free rows are nonzero
    assert torch.isfinite(y.float()).all()


@pytest.mark.parametrize("M,N,K,r", [(4096, 5120, 5120, 32), (1000, 15360, 5120, 64), (777, 5120, 13824, 64)])
def test_one_and_two_sm_kernels_agree_bitwise(M, N, K, r):
    """The 2-SM kernel changes the tiling, not the arithmetic: outputs equal the 1-SM kernel's bit for bit."""
    x = synthetic.activations(M, K, seed=31).to(DEV)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256).to(DEV)
    q, s = I.rotate_quant(x, 256)
    xa = I.lowrank_down(x, w.down)
    outs = []
    for mode in (1, 2):
        _lib.check(_lib.lib().convrot_set_gemm_mode(mode), "mode")
        try:
            outs.append((I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=w.up),
                         I.int8_mm_acc(q, w.qweight)))
        finally:
            _lib.lib().convrot_set_gemm_mode(0)
    assert torch.equal(outs[0][1], outs[1][1])
    # both kernels hold the dequantised values and add a separately computed low-rank product (its MMA over the
    # same K steps, 128 or 256 rows per instruction): the fused outputs are bitwise equal as well
    assert torch.equal(outs[0][0], outs[1][0])


def test_shared_lowrank_projection_matches_separate_layers(monkeypatch):
    """q/k/v with share_lowrank run one down projection over x and give the same outputs as separate layers."""
    kernels = I._kernels()
    calls = []
    down = kernels.lowrank_down
    monkeypatch.setattr(kernels, "lowrank_down", lambda *a: calls.append(a[1].shape[0]) or down(*a))

    def layer(seed):
        w = synthetic.linear_weights(1024, 512, rank=32, bias=True, group=256, seed_offset=seed)
        m = I.Int8RotLinear(1024, 512, 256, bias=True, rank=32)
        synthetic.load_into(m, w)
        return m.to(DEV)

    to_q, to_k, to_v = layer(0), layer(1), layer(2)
    x = synthetic.activations(300, 1024).to(DEV)
    separate = [to_q(x), to_k(x), to_v(x)]
    assert calls == [32, 32, 32]
    calls.clear()
    I.share_lowrank(to_q, to_k, to_v)
    to_q.keep_input = to_k.keep_input = True
    shared = [to_q(x), to_k(x), to_v(x)]
    assert calls == [96] and not I.Int8RotLinear._last_input
    for a, b in zip(separate, shared, strict=True):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M,K,N,r", [(333, 5120, 5120, 32), (17, 1024, 300, 0), (1024, 4096, 2048, 64)])
def test_convrot_linear_with_a_workspace_matches_the_module(M, K, N, r):
    """convrot_linear (C ABI: rotate+quantise into a caller workspace, then the GEMM) equals the module's calls."""
    import ctypes

    L = _lib.lib()
    x = synthetic.activations(M, K, seed=41).to(DEV)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256).to(DEV)
    nbytes = L.convrot_workspace_size(M, K, r)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=DEV)
    base = (ws.data_ptr() + 255) // 256 * 256
    ldy = -(-N // 8) * 8  # bf16 leading dimensions are multiples of 8 (16 bytes)
    y_full = torch.empty(M, ldy, dtype=torch.bfloat16, device=DEV)
    P = ctypes.c_void_p
    rc = L.convrot_linear(P(x.data_ptr()), K, P(w.qweight.data_ptr()), K, P(w.wscale.data_ptr()),
                          P(w.bias.data_ptr()), P(w.down.data_ptr()) if r else None, K,
                          P(w.up.data_ptr()) if r else None, r, r, M, N, K, 256, P(base), nbytes,
                          P(y_full.data_ptr()), ldy, P(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "convrot_linear")
    y = y_full[:, :N]
    # an odd leading dimension is refused, not written through
    assert L.convrot_linear(P(x.data_ptr()), K, P(w.qweight.data_ptr()), K, P(w.wscale.data_ptr()), None, None, 0,
                            None, 0, 0, M, N, K, 256, P(base), nbytes, P(y_full.data_ptr()), ldy + 1,
                            None) == (_lib.ERR_ALIGN if (ldy + 1) % 8 else _lib.OK)
    layer = I.Int8RotLinear(K, N, 256, bias=True, rank=r)
    synthetic.load_into(layer, w.to("cpu"))
    ref = layer.to(DEV)(x)
    if M >= I._MIN_KERNEL_ROWS:
        assert torch.equal(y, ref)
    else:  # the module reproduces the reference's torch-path rounding below 17 rows; the C entry does not
        assert close(y.float().cpu().numpy(), ref.float().cpu().numpy())[1] >= 0.9999


def pack(x: torch.Tensor, P: int) -> torch.Tensor:
    """[M, K] -> [P, M, K / P]: column block j of every row in [j] (the Ulysses all-to-all layout)."""
    M, K = x.shape
    return x.reshape(M, P, K // P).transpose(0, 1).contiguous()


@pytest.mark.parametrize("M,N,K,r,P", [
    (333, 5120, 5120, 32, 8), (4096, 2048, 1024, 0, 2), (1000, 1536, 512, 64, 4), (17, 640, 256, 16, 2),
])
def test_packed_gemm_output_is_the_plain_output_in_blocks(M, N, K, r, P, gemm_mode):
    """convrot_gemm_packed writes the same bits as convrot_gemm, column block j of each row to [j]."""
    x = synthetic.activations(M, K, seed=51).to(DEV)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256).to(DEV)
    q, s = I.rotate_quant(x, 256)
    xa = I.lowrank_down(x, w.down) if r else None
    up = w.up if r else None
    plain = I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=up)
    packed = I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=up, out_chunks=P)
    assert packed.shape == (P, M, N // P)
    assert torch.equal(packed, pack(plain, P))


@pytest.mark.parametrize("M,K,P,group", [(333, 5120, 8, 256), (1000, 4096, 2, 256), (64, 1024, 4, 64),
                                         (8, 5120, 8, 256), (16, 2048, 2, 16)])
def test_packed_rotate_and_down_projection_equal_the_plain_ones(M, K, P, group, rotate_variant):
    """The kernels reading the packed [P, M, K/P] receive layout give the plain layout's codes, scales and x.A."""
    x = synthetic.activations(M, K, seed=52).to(DEV)
    xp = pack(x, P)
    rounding = _lib.ROUND_KERNEL if M >= I._MIN_KERNEL_ROWS else _lib.ROUND_TORCH
    if rounding == _lib.ROUND_KERNEL:
        q, s = I.rotate_quant(x, group)
    else:
        q, s = I.rotate_quant_torch_rounding(x, group)
    qp, sp = I.rotate_quant_packed(xp, group, rounding)
    assert torch.equal(q, qp) and torch.equal(s, sp)
    down = synthetic.linear_weights(K, 64, rank=48, bias=False, group=256).down.to(DEV)
    assert torch.equal(I.lowrank_down(x, down), I.lowrank_down_packed(xp, down))


@pytest.mark.parametrize("M,K,N,r,P", [(333, 5120, 5120, 32, 8), (40, 1024, 2048, 0, 2), (9, 2048, 512, 16, 4)])
def test_layer_packed_forms_equal_the_plain_forward(M, K, N, r, P):
    """Int8RotLinear: forward(x, out_chunks=P) is forward(x) packed; forward_packed(pack(x)) is forward(x)."""
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256)
    layer = I.Int8RotLinear(K, N, 256, bias=True, rank=r)
    synthetic.load_into(layer, w)
    layer = layer.to(DEV)
    x = synthetic.activations(M, K, seed=53).to(DEV)
    ref = layer(x)
    assert torch.equal(layer(x, out_chunks=P), pack(ref, P))
    assert torch.equal(layer.forward_packed(pack(x, P)), ref)
    with pytest.raises(ValueError):
        layer.forward_packed(x)


@pytest.mark.parametrize("M,N,K,r,P", [(333, 5120, 5120, 32, 8), (4096, 2048, 1024, 0, 2), (40, 1536, 512, 64, 4)])
def test_scatter_gemm_writes_each_chunk_at_its_address(M, N, K, r, P, gemm_mode):
    """convrot_gemm_scatter with P separate buffers gives the packed output's blocks, bit for bit."""
    x = synthetic.activations(M, K, seed=61).to(DEV)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256).to(DEV)
    q, s = I.rotate_quant(x, 256)
    xa = I.lowrank_down(x, w.down) if r else None
    up = w.up if r else None
    packed = I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=up, out_chunks=P)
    W = N // P
    ld = W + 64  # rows of each destination further apart than the chunk: the pitch is honoured
    dests = [torch.full((M, ld), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(P)]
    assert I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=up,
                            out_ptrs=[t.data_ptr() for t in dests], out_ld=ld) is None
    for j in range(P):
        assert torch.equal(dests[j][:, :W], packed[j])
        assert torch.isnan(dests[j][:, W:].float()).all()  # nothing written past the chunk


@pytest.mark.parametrize("M,K,P,group", [(333, 5120, 8, 256), (1000, 4096, 2, 256), (64, 1024, 4, 64),
                                         (8, 5120, 8, 256)])
def test_gather_rotate_reads_rows_from_separate_chunks(M, K, P, group, rotate_variant):
    """convrot_rotate_quant_gather over P separate buffers equals rotate_quant of the plain rows; x_out is x."""
    x = synthetic.activations(M, K, seed=62).to(DEV)
    W = K // P
    ld = W + 128
    chunks = []
    for j in range(P):
        t = torch.zeros(M, ld, dtype=torch.bfloat16, device=DEV)
        t[:, :W] = x[:, j * W:(j + 1) * W]
        chunks.append(t)
    rounding = _lib.ROUND_KERNEL if M >= I._MIN_KERNEL_ROWS else _lib.ROUND_TORCH
    q, s = I.rotate_quant(x, group) if rounding == _lib.ROUND_KERNEL else I.rotate_quant_torch_rounding(x, group)
    qg, sg, xg = I.rotate_quant_gather([t.data_ptr() for t in chunks], ld, M, K, group, torch.device(DEV), rounding)
    assert torch.equal(q, qg) and torch.equal(s, sg)
    assert torch.equal(xg, x)


def test_layer_scatter_and_gather_forms_equal_the_plain_forward():
    """Int8RotLinear.forward_scatter / forward_gather on local buffers reproduce forward bit for bit."""
    K, N, r, M, P = 2048, 1024, 32, 300, 4
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256)
    layer = I.Int8RotLinear(K, N, 256, bias=True, rank=r)
    synthetic.load_into(layer, w)
    layer = layer.to(DEV)
    x = synthetic.activations(M, K, seed=63).to(DEV)
    ref = layer(x)
    outs = [torch.empty(M, N // P, dtype=torch.bfloat16, device=DEV) for _ in range(P)]
    layer.forward_scatter(x, [t.data_ptr() for t in outs], N // P)
    assert torch.equal(torch.cat(outs, dim=1), ref)
    chunks = [x[:, j * (K // P):(j + 1) * (K // P)].contiguous() for j in range(P)]
    assert torch.equal(layer.forward_gather([t.data_ptr() for t in chunks], M, K // P, x.device), ref)


def test_peer_wait_gives_up_at_its_limit_and_the_stream_goes_on():
    """A wait on a flag that nothing sets ends at the wait limit with CONVROT_ERR_TIMEOUT on the next poll; the
    stream is usable afterwards.  A flag that is set (here by this GPU's own signal kernel) passes."""
    import ctypes

    L = _lib.lib()
    flags = torch.zeros(8, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P_ = ctypes.c_void_p
    L.convrot_set_wait_limit_ns(50_000_000)  # 50 ms
    try:
        _lib.check(L.convrot_peer_wait(P_(flags.data_ptr()), 2, 1, stream), "wait")
        torch.cuda.synchronize()
        assert L.convrot_poll_error(None) == _lib.ERR_TIMEOUT
        slots = (ctypes.c_void_p * 2)(flags.data_ptr(), flags.data_ptr() + 4)
        _lib.check(L.convrot_peer_signal(slots, 2, 7, stream), "signal")
        _lib.check(L.convrot_peer_wait(P_(flags.data_ptr()), 2, 7, stream), "wait")
        _lib.check(L.convrot_peer_wait(P_(flags.data_ptr()), 2, 5, stream), "wait")  # already past: passes
        torch.cuda.synchronize()
        assert L.convrot_poll_error(None) == 0
        assert flags[:2].tolist() == [7, 7] and flags[2:].abs().sum().item() == 0
    finally:
        L.convrot_set_wait_limit_ns(2_000_000_000)
    assert L.convrot_peer_signal(None, 2, 1, stream) == _lib.ERR_ARG
    assert L.convrot_peer_wait(None, 2, 1, stream) == _lib.ERR_ARG


@pytest.mark.parametrize("M,K,N,r,bias", [(333, 5120, 27648, 64, True), (4096, 1024, 2048, 0, False),
                                          (17, 512, 1024, 32, True), (8, 2048, 512, 16, True)])
def test_fused_swiglu_is_bitwise_the_unfused_composition(M, K, N, r, bias, gemm_mode):
    """SwiGLUInt8 (the projection GEMM writing a * silu(g)) equals the projection followed by the bf16 torch ops
    on the GPU, and the oracle's restatement of those ops within one bf16 ulp."""
    from hyperflow_h3_flash_b200 import ffn

    w = synthetic.linear_weights(K, N, rank=r, bias=bias, group=256, seed_offset=7)
    proj = I.Int8RotLinear(K, N, 256, bias=bias, rank=r)
    synthetic.load_into(proj, w)
    proj = proj.to(DEV)
    fused = ffn.SwiGLUInt8(proj)
    x = synthetic.activations(M, K, seed=71).to(DEV)
    y = proj(x)
    ref = ffn.swiglu_reference(y)
    h = fused(x)
    assert h.shape == (M, N // 2)
    assert torch.equal(h, ref)
    orc = O.swiglu(bits(y))
    diff = np.abs(bits(h).astype(np.int32) - orc.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() >= 0.999


def test_epilogue_silu_is_torch_silu_on_every_bf16_input():
    """The SwiGLU epilogue's silu (its shared-memory table plus the formula for inputs outside it), run alone over
    all 65536 bf16 bit patterns, gives torch's F.silu bit for bit (NaN where torch gives NaN)."""
    from hyperflow_h3_flash_b200 import ffn

    x = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).to(DEV)
    y = ffn.silu_bf16(x)
    ref = F.silu(x)
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(y), nan)
    assert torch.equal(y.view(torch.int16)[~nan], ref.view(torch.int16)[~nan])
    # every pattern checked bitwise but the 254 NaN inputs and -inf (silu(-inf) = -inf / inf = NaN)
    assert int((~nan).sum()) == 65536 - 255


def test_fused_swiglu_outside_the_silu_table_is_still_bitwise(gemm_mode):
    """Projection outputs of magnitude zero, below 2^-19 or at least 32 are outside the epilogue's silu table and take
    the formula; the fused result is still the unfused composition bit for bit."""
    from hyperflow_h3_flash_b200 import ffn

    K, N, M = 1024, 1024, 300
    w = synthetic.linear_weights(K, N, rank=0, bias=False, group=256, seed_offset=9)
    ws = w.wscale.clone()
    ws[N // 2:N // 2 + 64] *= 1e-9  # g columns (the second half) with tiny magnitudes
    ws[N // 2 + 64:N // 2 + 128] *= 200.0  # and with large ones
    proj = I.Int8RotLinear(K, N, 256)
    proj.qweight.copy_(w.qweight)
    proj.wscale.copy_(ws)
    proj = proj.to(DEV)
    x = synthetic.activations(M, K, seed=73)
    x[5] = 0  # a zero row: g = 0 in every column
    x = x.to(DEV)
    y = proj(x)
    g = y[:, N // 2:].float()
    assert (g[:, :64].abs() < 2.0 ** -19).float().mean() > 0.5 and (g[:, 64:128].abs() >= 32).any()
    assert (g[5] == 0).all()
    assert torch.equal(ffn.SwiGLUInt8(proj)(x), ffn.swiglu_reference(y))


def test_fused_swiglu_gate_first_and_shape_checks():
    from hyperflow_h3_flash_b200 import ffn

    K, N = 1024, 512
    w = synthetic.linear_weights(K, N, rank=0, bias=False, group=256, seed_offset=8)
    proj = I.Int8RotLinear(K, N, 256)
    synthetic.load_into(proj, w)
    proj = proj.to(DEV)
    x = synthetic.activations(200, K, seed=72).to(DEV)
    assert torch.equal(ffn.SwiGLUInt8(proj, gate_first=True)(x), ffn.swiglu_reference(proj(x), gate_first=True))
    q, s = I.rotate_quant(x, 256)
    with pytest.raises(ValueError):
        I.convrot_matmul(q, proj.qweight[:480], s, proj.wscale[:480], swiglu=True)  # 480 % 64 != 0


def test_q_k_v_with_wide_ranks_fall_back_to_separate_down_projections():
    """share_lowrank on three rank-128 layers (384 > 256 outputs for one down GEMM) still gives the separate results."""
    def layer(seed):
        w = synthetic.linear_weights(512, 256, rank=128, bias=True, group=256, seed_offset=seed)
        m = I.Int8RotLinear(512, 256, 256, bias=True, rank=128)
        synthetic.load_into(m, w)
        return m.to(DEV)

    to_q, to_k, to_v = layer(0), layer(1), layer(2)
    x = synthetic.activations(200, 512, seed=81).to(DEV)
    separate = [to_q(x), to_k(x), to_v(x)]
    I.share_lowrank(to_q, to_k, to_v)
    to_q.keep_input = to_k.keep_input = True
    shared = [to_q(x), to_k(x), to_v(x)]
    for a, b in zip(separate, shared, strict=True):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M,K,T", [(333, 5120, 4), (4096, 2048, 1), (8, 1024, 2), (17, 256, 3)])
def test_adaln_prologue_is_the_oracle_and_quantises_its_own_h_bitwise(M, K, T):
    """The AdaLN rotate kernel's h equals the oracle's restatement (fp64 statistics; at most one bf16 ulp where the
    summation order moves a statistic's last bit), and its codes and scales are bitwise those of h."""
    g = torch.Generator().manual_seed(M + K)
    x = synthetic.activations(M, K, seed=91)
    scale = (torch.randn(T, K, generator=g) * 0.1).to(torch.bfloat16)
    shift = (torch.randn(T, K, generator=g) * 0.1).to(torch.bfloat16)
    idx = torch.randint(0, T, (M,), generator=g)
    rounding = _lib.ROUND_KERNEL if M >= I._MIN_KERNEL_ROWS else _lib.ROUND_TORCH
    q, s, h = I.rotate_quant_adaln(x.to(DEV), 256, scale.to(DEV), shift.to(DEV), idx.to(DEV), 1e-6, rounding)
    ref = O.adaln_modulate(bits(x), bits(scale), bits(shift), idx.numpy())
    diff = np.abs(bits(h).astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() >= 0.9999
    q_ref, s_ref = (O.rotate_quant if rounding == _lib.ROUND_KERNEL else O.rotate_quant_cpu)(bits(h), 256)
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)
    # and against the bf16 torch ops of chunk_block on the GPU (torch's own LayerNorm statistics)
    xd, sd, hd = x.to(DEV), scale.to(DEV), shift.to(DEV)
    tt = F.layer_norm(xd, (K,), eps=1e-6) * (1.0 + sd.index_select(0, idx.to(DEV)))
    th = tt + hd.index_select(0, idx.to(DEV))
    assert (h == th).float().mean().item() >= 0.995
    # torch's fp32 statistics (Welford mean, rsqrt) can move n by an ulp, which moves t = n * (1 + scale) by up to
    # two bf16 ulps, and t + shift can cancel: bound the difference by the final add's operands, not its result
    bound = (tt.float().abs() + hd.index_select(0, idx.to(DEV)).float().abs()) * 2.0**-5
    assert ((h.float() - th.float()).abs() <= bound).all()


def test_adaln_modulate_quantize_feeds_the_q_k_v_projections():
    """adaln_modulate_quantize leaves h's codes in the keep_input cache: q / k / v (with shared low-rank) give
    exactly what the same layers give on h computed without the cache, and no rotate kernel runs for them."""
    K, N, r, M = 1024, 512, 32, 300
    layers = []
    for i in range(3):
        w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256, seed_offset=30 + i)
        m = I.Int8RotLinear(K, N, 256, bias=True, rank=r)
        synthetic.load_into(m, w)
        layers.append(m.to(DEV))
    to_q, to_k, to_v = layers
    g = torch.Generator().manual_seed(5)
    x = synthetic.activations(M, K, seed=92).to(DEV)
    scale = (torch.randn(2, K, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    shift = (torch.randn(2, K, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    idx = (torch.arange(M) % 2).to(DEV)
    h = I.adaln_modulate_quantize(x, scale, shift, idx, 256)
    h_copy = h.clone()
    separate = [to_q(h_copy), to_k(h_copy), to_v(h_copy)]
    I.share_lowrank(to_q, to_k, to_v)
    to_q.keep_input = to_k.keep_input = True
    h = I.adaln_modulate_quantize(x, scale, shift, idx, 256)
    kernels = I._kernels()
    calls = []
    rq = kernels.rotate_quant
    kernels.rotate_quant = lambda *a: calls.append(1) or rq(*a)
    try:
        fused = [to_q(h), to_k(h), to_v(h)]
    finally:
        kernels.rotate_quant = rq
    assert calls == []
    for a, b in zip(separate, fused, strict=True):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M,K,N,r,T", [(333, 5120, 5120, 32, 4), (4096, 1024, 2048, 0, 1), (17, 512, 300, 64, 2),
                                        (8, 1024, 256, 16, 3)])
def test_gated_residual_epilogue_is_bitwise_the_bf16_composition(M, K, N, r, T, gemm_mode):
    """Int8RotLinear(x, residual=, gate=, gate_index=) equals `residual + gate[idx] * layer(x)` in bf16 torch ops."""
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256, seed_offset=40)
    layer = I.Int8RotLinear(K, N, 256, bias=True, rank=r)
    synthetic.load_into(layer, w)
    layer = layer.to(DEV)
    g = torch.Generator().manual_seed(M)
    x = synthetic.activations(M, K, seed=93).to(DEV)
    res = synthetic.activations(M, N, seed=94).to(DEV)
    gate = (torch.randn(T, N, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    idx = torch.randint(0, T, (M,), generator=g).to(DEV)
    y = layer(x)
    assert torch.equal(layer(x, residual=res, gate=gate, gate_index=idx), res + gate.index_select(0, idx) * y)
    assert torch.equal(layer(x, residual=res, gate=gate[0]), res + gate[0] * y)
    assert torch.equal(layer(x, residual=res), res + y)


def test_gated_residual_in_place_through_the_c_abi():
    """convrot_gemm_residual with y == res overwrites the residual stream with the result."""
    import ctypes

    M, K, N = 300, 1024, 512
    w = synthetic.linear_weights(K, N, rank=0, bias=False, group=256, seed_offset=41).to(DEV)
    x = synthetic.activations(M, K, seed=95).to(DEV)
    res = synthetic.activations(M, N, seed=96).to(DEV)
    gate = (torch.randn(2, N) * 0.3).to(torch.bfloat16).to(DEV)
    idx = (torch.arange(M) % 2).to(torch.int32).to(DEV)
    q, s = I.rotate_quant(x, 256)
    expected = res + gate.index_select(0, idx.long()) * I.convrot_matmul(q, w.qweight, s, w.wscale)
    P = ctypes.c_void_p
    buf = res.clone()
    rc = _lib.lib().convrot_gemm_residual(P(q.data_ptr()), K, P(w.qweight.data_ptr()), K, P(s.data_ptr()),
                                          P(w.wscale.data_ptr()), None, None, 0, None, 0, 0, M, N, K,
                                          P(buf.data_ptr()), N, P(gate.data_ptr()), N, P(idx.data_ptr()),
                                          P(buf.data_ptr()), N, P(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "convrot_gemm_residual")
    assert torch.equal(buf, expected)


def test_strided_row_views_go_to_the_kernels_uncopied_and_give_the_same_result():
    """A column slice of a wider tensor (v of a fused QKV output) is a strided row view: the layer reads it in place
    (row pitch passed to the kernels) and gives the bits of its contiguous copy; a transposed view is copied."""
    K, N, M = 1024, 512, 300
    w = synthetic.linear_weights(K, N, rank=32, bias=True, group=256, seed_offset=50)
    layer = I.Int8RotLinear(K, N, 256, bias=True, rank=32)
    synthetic.load_into(layer, w)
    layer = layer.to(DEV)
    wide = synthetic.activations(M, 3 * K, seed=97).to(DEV)
    view = wide[:, 2 * K:]
    assert view.stride() == (3 * K, 1)
    assert torch.equal(layer(view), layer(view.contiguous()))
    tr = view.contiguous().t().contiguous().t()  # same values, column-major
    assert torch.equal(layer(tr), layer(view.contiguous()))


def test_zero_padded_rank_gives_the_same_output():
    """The reference pads low-rank ranks with zero rows of down and zero columns of up at load
    (transformer.py:60-72, 205-216); the fused term over the padded rank is bitwise the unpadded one."""
    K, N, M, r = 1024, 512, 300, 40
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256, seed_offset=60)
    small = I.Int8RotLinear(K, N, 256, bias=True, rank=r)
    synthetic.load_into(small, w)
    padded = I.Int8RotLinear(K, N, 256, bias=True, rank=64)
    with torch.no_grad():
        padded.qweight.copy_(small.qweight)
        padded.wscale.copy_(small.wscale)
        padded.bias.copy_(small.bias)
        padded.down.weight.zero_()
        padded.up.weight.zero_()
        padded.down.weight[:r].copy_(small.down.weight)
        padded.up.weight[:, :r].copy_(small.up.weight)
    x = synthetic.activations(M, K, seed=98).to(DEV)
    assert torch.equal(small.to(DEV)(x), padded.to(DEV)(x))


@pytest.mark.parametrize("M,K,N", [(256, 4096, 5120), (333, 4096, 5120)])
def test_captured_graph_replays_the_layer_bitwise(M, K, N):
    """Config 5's cross-attention K/V projection captured once into a CUDA graph: replays on new inputs equal the
    eager layer bit for bit (and the two projections share one quantisation inside the graph)."""
    from hyperflow_h3_flash_b200.graphs import CapturedCall

    def layer(seed):
        w = synthetic.linear_weights(K, N, rank=32, bias=True, group=256, seed_offset=seed)
        m = I.Int8RotLinear(K, N, 256, bias=True, rank=32)
        synthetic.load_into(m, w)
        return m.to(DEV)

    to_k, to_v = layer(70), layer(71)
    to_k.keep_input = True

    def kv(x):
        return to_k(x), to_v(x)

    x0 = synthetic.activations(M, K, seed=99).to(DEV)
    graphed = CapturedCall(kv, x0)
    for seed in (100, 101):
        x = synthetic.activations(M, K, seed=seed).to(DEV)
        k_g, v_g = graphed(x)
        k_e, v_e = kv(x)
        assert torch.equal(k_g, k_e) and torch.equal(v_g, v_e)


@pytest.mark.parametrize("M,K,N,S,r,bias", [(40, 1024, 512, 3, 32, True), (333, 1024, 512, 2, 32, True),
                                             (4096, 1024, 512, 3, 0, False), (8, 1024, 512, 2, 64, True),
                                             (777, 1024, 768, 2, 48, True), (256, 4096, 5120, 2, 32, True)])
def test_grouped_layers_are_bitwise_the_separate_layers(M, K, N, S, r, bias, gemm_mode):
    """GroupedInt8RotLinear (one quantisation, one down projection, one GEMM launch writing each layer's output)
    gives each layer's own forward bit for bit, on the 1-SM and the 2-SM kernel; r = 48 makes a layer's rank chunk
    run past its xa columns into the next layer's, where its zero-filled up columns must cancel them exactly."""
    from hyperflow_h3_flash_b200.grouped import GroupedInt8RotLinear

    layers = []
    for s in range(S):
        w = synthetic.linear_weights(K, N, rank=r, bias=bias, group=256, seed_offset=90 + s)
        ly = I.Int8RotLinear(K, N, 256, bias=bias, rank=r)
        synthetic.load_into(ly, w)
        layers.append(ly.to(DEV))
    group = GroupedInt8RotLinear(*layers)
    x = synthetic.activations(M, K, seed=91).to(DEV)
    outs = group(x)
    assert len(outs) == S
    for ly, o in zip(layers, outs, strict=True):
        assert o.shape == (M, N)
        assert torch.equal(o, ly(x))


def test_grouped_layers_follow_weight_updates():
    from hyperflow_h3_flash_b200.grouped import GroupedInt8RotLinear

    layers = []
    for s in range(2):
        w = synthetic.linear_weights(512, 256, rank=16, bias=True, group=256, seed_offset=95 + s)
        ly = I.Int8RotLinear(512, 256, 256, bias=True, rank=16)
        synthetic.load_into(ly, w)
        layers.append(ly.to(DEV))
    group = GroupedInt8RotLinear(*layers)
    x = synthetic.activations(300, 512, seed=96).to(DEV)
    group(x)
    with torch.no_grad():
        layers[1].wscale.mul_(2.0)
        layers[0].up.weight.mul_(-1.0)
    outs = group(x)
    assert torch.equal(outs[0], layers[0](x)) and torch.equal(outs[1], layers[1](x))


def test_convrot_matmul_into_a_row_slice_equals_the_plain_result():
    """``out=`` (used by the chunked out projection) writes the plain result into rows of a larger buffer, bitwise,
    leaving the other rows alone; a wrong dtype, shape or column stride is refused."""
    M, K, N, r = 300, 1024, 512, 32
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256).to(DEV)
    x = synthetic.activations(M, K, seed=71).to(DEV)
    q, s = I.rotate_quant(x, 256)
    xa = I.lowrank_down(x, w.down)
    ref = I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=w.up)
    big = torch.full((M + 40, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    got = I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=w.up, out=big[16:16 + M])
    torch.cuda.synchronize()
    assert got.data_ptr() == big[16].data_ptr()
    assert torch.equal(big[16:16 + M], ref)
    assert torch.isnan(big[:16].float()).all() and torch.isnan(big[16 + M:].float()).all()
    for bad in (torch.empty(M, N - 8, dtype=torch.bfloat16, device=DEV),
                torch.empty(M, N, dtype=torch.float32, device=DEV),
                torch.empty(N, M, dtype=torch.bfloat16, device=DEV).t()):
        with pytest.raises(ValueError, match="out must be"):
            I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=w.up, out=bad)
