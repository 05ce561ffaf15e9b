"""Ulysses context parallelism around the convrot linears: token rows sharded over ranks, weights replicated.

The reference enables this with diffusers' ``ContextParallelConfig(ulysses_degree=P)``
(hyperflow_h3_flash, src/hyperflow_h3_flash/distributed.py:88-96); the all-to-all itself lives in diffusers.
Here it is written directly on ``torch.distributed.all_to_all_single`` (NCCL over NVLink on B200, gloo on CPU):

* every linear is token-wise, so each rank runs its ``M / P`` rows with no communication;
* around attention, ``seq_to_head`` turns ``[M/P, H, D]`` (local tokens, all heads) into ``[M, H/P, D]`` (all tokens,
  local heads) and ``head_to_seq`` is its inverse.  The head count must be divisible by ``P``
  (distributed.py:68-71).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


def world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def shard_rows(x: Tensor, world_size: int, rank: int) -> Tensor:
    """This rank's contiguous slice of the token rows (rows must divide evenly)."""
    M = x.shape[0]
    if M % world_size:
        raise ValueError(f"{M} token rows do not split evenly over {world_size} ranks")
    step = M // world_size
    return x[rank * step : (rank + 1) * step]


def seq_to_head(t: Tensor, heads: int, group=None) -> Tensor:
    """``[M/P, heads * D]`` on every rank -> ``[M, heads/P, D]``: all tokens of this rank's heads."""
    P = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
    m, width = t.shape
    if heads % P or width % heads:
        raise ValueError(f"{heads} heads of width {width // max(heads, 1)} cannot split over {P} ranks")
    d = width // heads
    if P == 1:
        return t.reshape(m, heads, d)
    send = t.reshape(m, P, heads // P, d).transpose(0, 1).contiguous()  # [P, m, H/P, D]: chunk j -> rank j
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)  # chunk i <- rank i's tokens
    return recv.reshape(P * m, heads // P, d)


def head_to_seq(t: Tensor, group=None) -> Tensor:
    """Inverse of ``seq_to_head``: ``[M, H/P, D]`` -> ``[M/P, H * D]``."""
    P = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
    M, hp, d = t.shape
    if P == 1:
        return t.reshape(M, hp * d)
    if M % P:
        raise ValueError(f"{M} tokens do not split over {P} ranks")
    m = M // P
    send = t.reshape(P, m, hp, d).contiguous()  # chunk i -> rank i (its tokens)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)  # chunk j <- rank j's heads
    return recv.transpose(0, 1).reshape(m, P * hp * d)


def _packed_capable(x: Tensor, layers) -> bool:
    return x.is_cuda and all(hasattr(layer, "forward_packed") for layer in layers)


def attention_block_linears(x: Tensor, to_q, to_k, to_v, to_out, heads: int, attention=None, group=None) -> Tensor:
    """One attention block's linears on this rank's tokens: q/k/v (sharing one quantisation -- and one low-rank
    projection, see ``int8.share_lowrank`` -- when the layers have ``keep_input``), the seq->head all-to-all,
    ``attention`` (identity -> v when None), head->seq, and ``to_out``.

    With convrot layers on CUDA and more than one rank, the q/k/v GEMMs write their outputs straight into the
    all-to-all send layout ``[P, M/P, heads/P * D]`` and ``to_out`` reads the receive layout in place, so no pack
    or unpack copy surrounds the collectives; each q/k/v all-to-all is issued as soon as its GEMM is queued and
    overlaps the next GEMM."""
    P = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
    if P == 1 or not _packed_capable(x, (to_q, to_k, to_v, to_out)):
        q, k, v = to_q(x), to_k(x), to_v(x)
        qh, kh, vh = seq_to_head(q, heads, group), seq_to_head(k, heads, group), seq_to_head(v, heads, group)
        oh = vh if attention is None else attention(qh, kh, vh)
        return to_out(head_to_seq(oh, group))
    m = x.reshape(-1, x.shape[-1]).shape[0]
    width = to_q.out_features
    if heads % P or width % heads:
        raise ValueError(f"{heads} heads cannot split over {P} ranks")
    d = width // heads
    received, works = [], []
    for layer in (to_q, to_k, to_v):
        send = layer(x, out_chunks=P)  # [P, m, width / P]: block j is rank j's heads
        recv = torch.empty_like(send)
        works.append(dist.all_to_all_single(recv, send, group=group, async_op=True))
        received.append(recv)
    for work in works:
        work.wait()
    qh, kh, vh = (t.reshape(P * m, heads // P, d) for t in received)  # every token of this rank's heads
    oh = vh if attention is None else attention(qh, kh, vh)
    send = oh.reshape(P, m, (heads // P) * d).contiguous()  # block i: the tokens of rank i
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)  # block j: this rank's tokens, heads of rank j
    return to_out.forward_packed(recv)
