"""convrot_linear_noalloc: the whole layer for callers that cannot allocate device memory on the call path.

Some callers own every byte of device memory themselves: serving runtimes plan a fixed arena at start-up and
forbid later allocations, plugin-style interfaces hand over only the inputs, the outputs and a stream, and latency
sensitive code avoids cudaMalloc / cudaFree because they can synchronise the device.  For them the library offers
one entry point that keeps its intermediates (codes, scales, low-rank input) in scratch built into the library
instead of a caller workspace.  Here it is called through the C ABI and compared with convrot_linear, which runs
the same kernels on a caller-provided workspace: the outputs must be bitwise equal, on two calls in a row whose
inputs differ (the built-in scratch keeps the previous call's contents, which must not leak into the next).

This file is named to be collected last, so a run that stops at its first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from hyperflow_h3_flash_b200 import _lib
from hyperflow_h3_flash_b200 import synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"
P = ctypes.c_void_p


def _ptr(t):
    return None if t is None else P(t.data_ptr())


def _up_padded(w, r):
    """LowRankLinear.up's weight [N, r] with its rows padded to a multiple of 8 elements (the 16-byte rule of the
    C ABI's leading dimensions), and that leading dimension."""
    ld_up = -(-r // 8) * 8
    if ld_up == r:
        return w.up, r
    up = torch.zeros(w.up.shape[0], ld_up, dtype=w.up.dtype, device=w.up.device)
    up[:, :r] = w.up
    return up, ld_up


def _with_workspace(L, x, w, r, group):
    """The existing entry point: convrot_linear on a workspace allocated by the caller (here: torch)."""
    M, K = x.shape
    N = w.qweight.shape[0]
    up, ld_up = _up_padded(w, r) if r else (None, 0)
    nbytes = L.convrot_workspace_size(M, K, r)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=DEV)
    base = (ws.data_ptr() + 255) // 256 * 256
    y = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    rc = L.convrot_linear(_ptr(x), K, _ptr(w.qweight), K, _ptr(w.wscale), _ptr(w.bias),
                          _ptr(w.down) if r else None, K, _ptr(up), ld_up, r, M, N, K, group,
                          P(base), nbytes, _ptr(y), N, P(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "convrot_linear")
    return y


def _no_alloc(L, x, w, r, group):
    M, K = x.shape
    N = w.qweight.shape[0]
    up, ld_up = _up_padded(w, r) if r else (None, 0)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    rc = L.convrot_linear_noalloc(_ptr(x), K, _ptr(w.qweight), K, _ptr(w.wscale), _ptr(w.bias),
                                  _ptr(w.down) if r else None, K, _ptr(up), ld_up, r, M, N, K, group,
                                  _ptr(y), N, P(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "convrot_linear_noalloc")
    return y


def _largest_rows_that_fit(L, K, r):
    """The largest M whose codes, scales and low-rank input (convrot_workspace_size) fit the built-in scratch."""
    lo, hi = 1, 1 << 20  # fits / does not fit
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if L.convrot_workspace_size(mid, K, r) <= _lib.NOALLOC_SCRATCH_BYTES:
            lo = mid
        else:
            hi = mid
    return lo


def test_no_alloc_entry_matches_the_workspace_entry_on_two_calls_in_a_row():
    L = _lib.lib()
    cases = [  # (M, K, N, r, group, seed): each call is smaller than the one before, so stale scratch would show
        (1000, 5120, 2048, 32, 256, 1),
        (333, 4096, 1536, 64, 256, 2),
        (77, 1024, 512, 36, 256, 4),  # a rank that is not a multiple of 8 (xa rows padded inside the scratch)
    ]
    for M, K, N, r, group, seed in cases:
        x = synthetic.activations(M, K, seed=seed).to(DEV)
        w = synthetic.linear_weights(K, N, rank=r, bias=True, group=group, seed_offset=seed).to(DEV)
        expected = _with_workspace(L, x, w, r, group)
        got = _no_alloc(L, x, w, r, group)
        torch.cuda.synchronize()
        # the tolerance of this repository's parity tests for the same kernels: bitwise
        assert torch.equal(got, expected), (M, K, N, r)
    assert L.convrot_poll_error(None) == 0


def test_no_alloc_entry_without_low_rank_and_its_size_limit():
    L = _lib.lib()
    x = synthetic.activations(64, 1024, seed=3).to(DEV)
    w = synthetic.linear_weights(1024, 512, rank=0, bias=False, group=256).to(DEV)
    assert torch.equal(_no_alloc(L, x, w, 0, 256), _with_workspace(L, x, w, 0, 256))
    # beyond the built-in scratch: rejected before anything is launched (null pointers are never touched)
    M, K = 8192, 5120  # 40 MiB of codes
    rc = L.convrot_linear_noalloc(P(16), K, P(16), K, P(16), None, None, 0, None, 0, 0, M, 512, K, 256, P(16),
                                  512, None)
    assert rc == _lib.ERR_SCRATCH
    assert "scratch" in _lib.status_string(rc)
    assert _lib.NOALLOC_SCRATCH_BYTES == 16 << 20


def test_no_alloc_entry_at_the_edge_of_its_scratch():
    """The largest problem that fits the scratch (K = 5120, r = 32) runs and equals the workspace entry bitwise;
    one more row is rejected before anything is launched."""
    L = _lib.lib()
    K, N, r = 5120, 512, 32
    M = _largest_rows_that_fit(L, K, r)
    assert L.convrot_workspace_size(M + 1, K, r) > _lib.NOALLOC_SCRATCH_BYTES >= L.convrot_workspace_size(M, K, r)
    x = synthetic.activations(M, K, seed=5).to(DEV)
    w = synthetic.linear_weights(K, N, rank=r, bias=True, group=256, seed_offset=5).to(DEV)
    got = _no_alloc(L, x, w, r, 256)
    expected = _with_workspace(L, x, w, r, 256)
    torch.cuda.synchronize()
    assert torch.equal(got, expected)
    rc = L.convrot_linear_noalloc(P(16), K, P(16), K, P(16), None, P(16), K, P(16), r, r, M + 1, N, K, 256, P(16),
                                  N, None)
    assert rc == _lib.ERR_SCRATCH
    assert L.convrot_poll_error(None) == 0
