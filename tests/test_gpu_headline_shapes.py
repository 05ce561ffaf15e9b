"""The fused layer at the headline shapes, on launches where every CTA pair runs many tiles, against the oracle.

These are the launches the bench times: config 2 (M = 32768, K = N = 5120, r = 32) and config 3's four linears at
M = 32760 with r = 64 (QKV 5120 -> 15360, out 5120 -> 5120, FFN-up 5120 -> 27648 with and without the SwiGLU
epilogue, FFN-down 13824 -> 5120), all with bias, on both GEMM kernels.  At these sizes each of the 74 CTA pairs
(148 CTAs of the 1-SM kernel) loops over tens of tiles, so the double-buffered accumulators, the low-rank barriers'
alternating phases and the ragged last tile all take part.  The whole output is computed; 64 rows are checked
against the oracle's fused layer (int8.py:161-171 kernel arithmetic + bias + up(down(x)), transformer.py:57-58):
the first rows, rows of the last (ragged) tile, and random rows.

Bit-exact: codes, scales and the int32 accumulator of the sampled rows.  The fused output (no reference counterpart)
within the north-star tolerance -- max |err| / max |ref| <= 1e-2 and cosine >= 0.9999 -- and every value within two
bf16 ulps (|err| <= |ref| 2^-6 + 1e-3 max |ref|) of the oracle's value.
"""

from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from hyperflow_h3_flash_b200 import _lib
from hyperflow_h3_flash_b200 import int8 as I
from hyperflow_h3_flash_b200 import synthetic
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
G = 256


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def sample_rows(M: int, seed: int) -> np.ndarray:
    """64 rows: the first 8, the last 24 (inside the last, ragged 256-row pair tile), 32 random ones."""
    rng = np.random.default_rng(seed)
    picked = set(range(8)) | set(range(M - 24, M))
    while len(picked) < 64:
        picked.add(int(rng.integers(8, M - 24)))
    return np.array(sorted(picked))


def check_fused(out: np.ndarray, ref_bits: np.ndarray) -> None:
    ref = O.bf16_to_f32(ref_bits).astype(np.float64)
    out = out.astype(np.float64)
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    cos = (out * ref).sum() / np.sqrt((out * out).sum() * (ref * ref).sum())
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    bound = np.abs(ref) * 2.0**-6 + 1e-3 * np.abs(ref).max()
    assert (np.abs(out - ref) <= bound).all(), float((np.abs(out - ref) / np.maximum(bound, 1e-30)).max())


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.lib().convrot_poll_error(None) == 0


@pytest.fixture(params=[1, 2], ids=["gemm1sm", "gemm2sm"])
def gemm_mode(request):
    _lib.check(_lib.lib().convrot_set_gemm_mode(request.param), "gemm mode")
    yield request.param
    _lib.lib().convrot_set_gemm_mode(0)


CASES = {  # name: (M, K, N, r)
    "cfg2": (32768, 5120, 5120, 32),
    "cfg3_qkv": (32760, 5120, 15360, 64),
    "cfg3_out": (32760, 5120, 5120, 64),
    "cfg3_ffn_up": (32760, 5120, 27648, 64),
    "cfg3_ffn_down": (32760, 13824, 5120, 64),
}


@functools.cache
def case_inputs(M: int, K: int, N: int, r: int, seed: int):
    """Inputs and weights of one case, built once for both GEMM kernels (synthesising a 141 MB weight takes a
    while on the CPU)."""
    return (synthetic.activations(M, K, seed=seed),
            synthetic.linear_weights(K, N, rank=r, bias=True, group=G, seed_offset=seed))


@pytest.mark.parametrize("name", list(CASES))
def test_fused_layer_at_headline_shapes_matches_the_oracle(name, gemm_mode):
    M, K, N, r = CASES[name]
    seed = sorted(CASES).index(name)
    x, w = case_inputs(M, K, N, r, 40 + seed)
    layer = I.Int8RotLinear(K, N, G, bias=True, rank=r)
    synthetic.load_into(layer, w)
    layer = layer.to(DEV)
    xd = x.to(DEV)
    y = layer(xd)
    q, s = I.rotate_quant(xd, G)
    rows = sample_rows(M, seed)
    acc = I.int8_mm_acc(q[torch.from_numpy(rows).to(DEV)], layer.qweight)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    orc = O.convrot_linear(bits(x[rows]), w.qweight.numpy(), w.wscale.numpy(), G, bits(w.bias),
                           bits(w.down.t().contiguous()), bits(w.up.t().contiguous()))
    assert np.array_equal(q[rows].cpu().numpy(), orc["q"])
    assert np.array_equal(s[rows].cpu().numpy(), orc["s"])
    assert np.array_equal(acc.cpu().numpy(), orc["acc"])
    check_fused(y[rows].float().cpu().numpy(), orc["out"])


def test_fused_swiglu_ffn_up_at_the_block_shape_matches_the_oracle(gemm_mode):
    """Config 3's FFN-up (M = 32760, 5120 -> 27648, r = 64, bias) with the SwiGLU epilogue: h = a * silu(g) of the
    sampled rows against the oracle's swiglu of its fused projection rows."""
    from hyperflow_h3_flash_b200 import ffn

    M, K, N, r = CASES["cfg3_ffn_up"]
    x, w = case_inputs(M, K, N, r, 40 + sorted(CASES).index("cfg3_ffn_up"))
    proj = I.Int8RotLinear(K, N, G, bias=True, rank=r)
    synthetic.load_into(proj, w)
    fused = ffn.SwiGLUInt8(proj.to(DEV))
    h = fused(x.to(DEV))
    torch.cuda.synchronize()
    assert h.shape == (M, N // 2)
    rows = sample_rows(M, 7)
    orc = O.convrot_linear(bits(x[rows]), w.qweight.numpy(), w.wscale.numpy(), G, bits(w.bias),
                           bits(w.down.t().contiguous()), bits(w.up.t().contiguous()))
    check_fused(h[torch.from_numpy(rows).to(DEV)].float().cpu().numpy(), O.swiglu(orc["out"]))
