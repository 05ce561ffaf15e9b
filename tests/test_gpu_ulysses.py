"""The Ulysses attention-block linears on two GPUs: NCCL with the packed layouts, and the peer-memory exchange.

With more than one rank, ``ulysses.attention_block_linears`` lets the q/k/v GEMMs write the all-to-all send layout
directly and the out projection read the receive layout in place; with a ``PeerExchange`` the GEMMs store into the
other GPU's receive buffers and the out projection's rotate kernel reads from them.  Every step of either path is
exact (the GEMM outputs are bitwise those of the plain layout, the exchanges are permutations), so each rank's
result must equal, bit for bit, the same token-wise computation on its own rows with no communication.  Skipped on fewer than two GPUs;
ranks are spawned processes with a file store, as in the CPU tests of the same module.
"""

from __future__ import annotations

import datetime

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HEADS, K, RANK_LR, ROWS = 8, 1024, 16, 300


def _layers(dev):
    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic

    layers = []
    for i in range(4):
        w = synthetic.linear_weights(K, K, rank=RANK_LR, bias=True, group=256, seed_offset=i)
        layer = I.Int8RotLinear(K, K, 256, bias=True, rank=RANK_LR)
        synthetic.load_into(layer, w)
        layers.append(layer.to(dev))
    return layers


def _worker(rank, world, store_path, out_path):
    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic, ulysses

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{store_path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        to_q, to_k, to_v, to_out = _layers(dev)
        x = synthetic.activations(ROWS, K, seed=100 + rank).to(dev)
        with torch.inference_mode():
            # reference first: plain token-wise layers on this rank's rows, no communication
            ref_v = to_out(to_v(x))
            ref_qkv = to_out(to_q(x) + to_k(x) + to_v(x))
            to_q.keep_input = to_k.keep_input = True
            I.share_lowrank(to_q, to_k, to_v)
            out_v = ulysses.attention_block_linears(x, to_q, to_k, to_v, to_out, HEADS)
            out_qkv = ulysses.attention_block_linears(x, to_q, to_k, to_v, to_out, HEADS,
                                                      attention=lambda q, k, v: q + k + v)
            torch.cuda.synchronize()
        res = {"identity": torch.equal(out_v, ref_v), "sum": torch.equal(out_qkv, ref_qkv),
               "shape": tuple(out_v.shape) == (ROWS, K)}
        torch.save(res, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def _worker_peer(rank, world, store_path, out_path, copy_names, pull_chunks=0):
    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic, ulysses

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{store_path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    ex = None
    try:
        to_q, to_k, to_v, to_out = _layers(dev)
        ex = ulysses.PeerExchange(ROWS, K, HEADS, device=dev, copy_names=copy_names, pull_chunks=pull_chunks)
        res = {}
        with torch.inference_mode():
            for step in range(3):  # the buffers and flags are reused step after step
                x = synthetic.activations(ROWS, K, seed=200 + 10 * step + rank).to(dev)
                I.Int8RotLinear._last_input.clear()
                ref_v = to_out(to_v(x))
                ref_qkv = to_out(to_q(x) + to_k(x) + to_v(x))
                out_v = ulysses.attention_block_linears(x, to_q, to_k, to_v, to_out, HEADS, exchange=ex)
                out_qkv = ulysses.attention_block_linears(x, to_q, to_k, to_v, to_out, HEADS, exchange=ex,
                                                          attention=lambda q, k, v: q + k + v)
                torch.cuda.synchronize()
                res[f"identity{step}"] = torch.equal(out_v, ref_v)
                res[f"sum{step}"] = torch.equal(out_qkv, ref_qkv)
        res["poll"] = I._lib.lib().convrot_poll_error(None)
        torch.save(res, f"{out_path}.{rank}")
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("copy_names,pull_chunks", [(("q", "k"), 0), ((), 0), ((), 3)],
                         ids=["copy_engines_qk", "epilogue_stores_only", "out_projection_pulled_in_3_chunks"])
def test_peer_memory_exchange_on_two_gpus_equals_the_local_computation(tmp_path, copy_names, pull_chunks):
    """The exchange over peer memory (GEMM stores into the other GPU, or local writes moved by the copy engines;
    the rotate kernel reads from the other GPU, or the copy engines pull the out projection's input in row chunks)
    is bitwise the local computation, step after step."""
    world = 2
    mp.spawn(_worker_peer, args=(world, str(tmp_path / "store"), str(tmp_path / "out"), copy_names, pull_chunks),
             nprocs=world, join=True)
    for rank in range(world):
        res = torch.load(f"{tmp_path / 'out'}.{rank}")
        assert all(v is True for k, v in res.items() if k != "poll"), (rank, res)
        assert res["poll"] == 0, (rank, res)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_packed_attention_block_on_two_gpus_equals_the_local_computation(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, str(tmp_path / "store"), str(tmp_path / "out")), nprocs=world, join=True)
    for rank in range(world):
        res = torch.load(f"{tmp_path / 'out'}.{rank}")
        assert res == {"identity": True, "sum": True, "shape": True}, (rank, res)
