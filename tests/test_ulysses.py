"""Ulysses token sharding and the seq<->head all-to-all on CPU ranks (gloo, world size 2), in the pattern of the
reference's distributed tests (tests/test_distributed.py:67-71, 153-166: file store, mp.spawn, bitwise checks).

The all-to-all is a pure permutation (its third-party original in diffusers has no test in the reference), so it is
pinned here: the round trip is the identity, the head split is the expected slice of the gathered tensor, and a
token-wise pipeline on two ranks gives the single-rank result bitwise.  A rank that dies is reported, not hung on.
"""

from __future__ import annotations

import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hyperflow_h3_flash_b200 import ulysses

HEADS, D = 8, 4


def _init(rank, world, store_path):
    dist.init_process_group("gloo", init_method=f"file://{store_path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    torch.set_num_threads(2)


def _global_tokens(M):
    g = torch.Generator().manual_seed(0)
    return torch.randn(M, HEADS * D, generator=g)


def _worker_roundtrip(rank, world, store_path, out_path):
    _init(rank, world, store_path)
    try:
        M = 12
        full = _global_tokens(M)
        local = ulysses.shard_rows(full, world, rank)
        heads = ulysses.seq_to_head(local, HEADS)
        # this rank holds every token of heads [rank*H/P, (rank+1)*H/P)
        expect = full.reshape(M, HEADS, D)[:, rank * HEADS // world:(rank + 1) * HEADS // world]
        ok_heads = torch.equal(heads, expect)
        back = ulysses.head_to_seq(heads)
        ok_back = torch.equal(back, local)

        # a token-wise pipeline (two linears around an identity attention) equals the single-rank pipeline bitwise
        w1 = torch.randn(HEADS * D, HEADS * D, generator=torch.Generator().manual_seed(1))
        w2 = torch.randn(HEADS * D, HEADS * D, generator=torch.Generator().manual_seed(2))
        lin1 = lambda t: t @ w1  # noqa: E731
        lin2 = lambda t: t @ w2  # noqa: E731
        out = ulysses.attention_block_linears(local, lin1, lin1, lin1, lin2, HEADS)
        ref = ulysses.shard_rows(lin2(lin1(full)), world, rank)
        ok_pipe = torch.allclose(out, ref, rtol=0, atol=0) or torch.equal(out, ref)
        torch.save({"heads": ok_heads, "back": ok_back, "pipe": ok_pipe}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_all_to_all_round_trip_and_pipeline_on_two_cpu_ranks(tmp_path):
    world = 2
    store = tmp_path / "store"
    out = tmp_path / "out"
    mp.spawn(_worker_roundtrip, args=(world, str(store), str(out)), nprocs=world, join=True)
    for rank in range(world):
        res = torch.load(f"{out}.{rank}")
        assert res == {"heads": True, "back": True, "pipe": True}, (rank, res)


def _worker_dies(rank, world, store_path, out_path):
    _init(rank, world, store_path)
    if rank == 1:
        os._exit(3)  # leaves between steps, with nothing in flight
    try:
        local = torch.randn(4, HEADS * D)
        ulysses.seq_to_head(local, HEADS)
        result = "completed"
    except Exception as e:  # gloo reports the lost peer instead of waiting forever
        result = type(e).__name__
    torch.save(result, f"{out_path}.{rank}")


def test_a_lost_rank_surfaces_as_an_error(tmp_path):
    world = 2
    ctx = mp.start_processes(_worker_dies, args=(world, str(tmp_path / "store"), str(tmp_path / "out")),
                             nprocs=world, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in ctx.processes)
    res = torch.load(f"{tmp_path / 'out'}.0")
    assert res != "completed"


def test_shapes_are_checked():
    with pytest.raises(ValueError):
        ulysses.shard_rows(torch.zeros(5, 4), 2, 0)
    t = torch.zeros(6, HEADS * D)
    assert ulysses.seq_to_head(t, HEADS).shape == (6, HEADS, D)  # single process: no exchange
    assert ulysses.head_to_seq(ulysses.seq_to_head(t, HEADS)).shape == (6, HEADS * D)


def _worker_exchange_setup_fails(rank, world, store_path, out_path):
    _init(rank, world, store_path)
    try:
        # host memory cannot be exported through CUDA IPC: every rank must get the error, none may hang
        ulysses.PeerExchange(16, 8 * 128, 8, device=torch.device("cpu"))
        result = "constructed"
    except RuntimeError as e:
        result = str(e)
    finally:
        dist.destroy_process_group()
    torch.save(result, f"{out_path}.{rank}")


def test_peer_exchange_setup_failure_reaches_every_rank(tmp_path):
    world = 2
    ctx = mp.start_processes(_worker_exchange_setup_fails, args=(world, str(tmp_path / "store"), str(tmp_path / "out")),
                             nprocs=world, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in ctx.processes)
    for rank in range(world):
        assert "could not export" in torch.load(f"{tmp_path / 'out'}.{rank}")
