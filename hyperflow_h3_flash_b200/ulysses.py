"""Ulysses context parallelism around the convrot linears: token rows sharded over ranks, weights replicated.

The reference enables this with diffusers' ``ContextParallelConfig(ulysses_degree=P)``
(hyperflow_h3_flash, src/hyperflow_h3_flash/distributed.py:88-96); the all-to-all itself lives in diffusers.
Here it is written directly on ``torch.distributed.all_to_all_single`` (NCCL over NVLink on B200, gloo on CPU):

* every linear is token-wise, so each rank runs its ``M / P`` rows with no communication;
* around attention, ``seq_to_head`` turns ``[M/P, H, D]`` (local tokens, all heads) into ``[M, H/P, D]`` (all tokens,
  local heads) and ``head_to_seq`` is its inverse.  The head count must be divisible by ``P``
  (distributed.py:68-71).
* ``PeerExchange`` does the same exchange without a collective: the producing GEMM stores into the other GPUs'
  receive buffers and the consuming rotate kernel reads from them, ordered by epoch flags.
"""

from __future__ import annotations

import ctypes

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


class PeerExchange:
    """The Ulysses exchange over peer memory: this rank's receive buffers, mapped by every rank of the group.

    The buffers live in this GPU's memory; every other rank maps them through CUDA IPC (one process per GPU), so
    the q/k/v GEMMs of rank i store column block j of their outputs straight into rank j's receive buffer, slot i
    (``convrot_gemm_scatter``), and the out projection's rotate kernel of rank i reads block i of every rank's
    attention output straight from that rank's memory (``convrot_rotate_quant_gather``): the bytes cross NVLink
    inside the kernels that produce and consume them.  Layers named in ``copy_names`` instead write their output
    locally in the send layout and the GPU's copy engines move the blocks into the other ranks' buffers on a stream
    of their own, overlapping the next GEMM (``convrot_copy_blocks``).  Measured on 2 B200s that is slower (3.44
    against 3.15 ms per config-2 step with q and k copied: the copies contend with the next GEMM for HBM and
    NVLink), so the default is none.  No collective library either way.

    Ordering is two epoch flags per step (``convrot_peer_signal`` / ``convrot_peer_wait``, release/acquire at
    system scope, bounded waits):

    * ARRIVED -- rank i has written its q/k/v blocks into every rank.  Rank j waits for all ranks before attention.
    * READY   -- rank j's attention output is complete.  Rank i waits for all ranks before gathering.

    Those two also cover reuse across steps: rank i writes rank j's receive buffers of step s+1 only after READY(s)
    from rank j (so j's attention of step s is done reading them), and rank j overwrites its attention output of
    step s+1 only after ARRIVED(s+1) from rank i, which rank i signals after its gather of step s.

    Layout of each rank's buffer: 4 KiB of flags (phase p, source rank i at word ``8 p + i``), then the receive
    buffers q, k, v and the attention output, each ``[P, rows, width / P]`` bf16 (block i: rank i's tokens).
    """

    ARRIVED, READY = 0, 1
    _NAMES = ("q", "k", "v", "out")
    _FLAG_BYTES = 4096

    def __init__(self, rows: int, width: int, heads: int, group=None, device: torch.device | None = None,
                 copy_names: tuple[str, ...] = (), pull_chunks: int = 0):
        from . import _lib

        self._lib = _lib
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.P > 8 or heads % self.P or width % heads or (width // self.P) % 128:
            raise ValueError(f"{heads} heads of width {width} cannot be exchanged over {self.P} ranks")
        self.rows, self.width, self.heads = rows, width, heads
        self.W = width // self.P
        # pull_chunks = n > 0: the out projection's input is pulled by the copy engines in n row chunks into a local
        # staging buffer, each chunk overlapping the previous chunk's out projection (see attention_block_peer)
        self.pull_chunks = int(pull_chunks)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._tensor_bytes = self.P * rows * self.W * 2
        self.buf = torch.zeros(self._FLAG_BYTES + len(self._NAMES) * self._tensor_bytes, dtype=torch.uint8,
                               device=self.device)
        L = _lib.lib()
        # Every rank takes the same collective steps whether or not its own part fails, so a failure on one rank
        # raises on all of them instead of leaving the others waiting.
        handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        offset = ctypes.c_int64(0)
        rc = L.convrot_ipc_handle(ctypes.c_void_p(self.buf.data_ptr()), handle, ctypes.byref(offset))
        everyone: list = [None] * self.P
        dist.all_gather_object(everyone, (handle.raw, offset.value) if rc == _lib.OK else None, group=group)
        if any(e is None for e in everyone):
            raise RuntimeError("a rank could not export its exchange buffer (CUDA IPC)")
        self._opened: list[int] = []
        self.base: list[int] = []
        error = None
        for j, (h, off) in enumerate(everyone):
            if j == self.rank:
                self.base.append(self.buf.data_ptr())
                continue
            mapped = ctypes.c_void_p(0)
            rc = L.convrot_ipc_open(ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES), ctypes.byref(mapped))
            if rc != _lib.OK:
                error = f"convrot_ipc_open of rank {j}: {_lib.status_string(rc)}"
                break
            self._opened.append(mapped.value)
            self.base.append(mapped.value + off)
        failed = torch.tensor([0 if error is None else 1], device=self.device)
        dist.all_reduce(failed, group=group)
        if failed.item():
            self._unmap()
            raise RuntimeError(error or "another rank could not map the exchange buffers")
        self.epoch = 0
        self.kernel_launches = 0
        # Layers (of "q", "k", "v") whose output is written locally in the send layout and then moved into the
        # other GPUs' receive buffers by the copy engines, on their own stream, while the next GEMM runs; the rest
        # store straight into the other GPUs' buffers from the GEMM epilogue.
        if any(n not in ("q", "k", "v") for n in copy_names):
            raise ValueError(f"copy_names must name q, k or v, got {copy_names!r}")
        self.copy_names = tuple(copy_names)
        self.copy_stream = torch.cuda.Stream(self.device)
        self.pull_stage = (torch.empty(self.P, rows, self.W, dtype=torch.bfloat16, device=self.device)
                           if self.pull_chunks > 0 else None)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def _offset(self, name: str) -> int:
        return self._FLAG_BYTES + self._NAMES.index(name) * self._tensor_bytes

    def recv(self, name: str) -> Tensor:
        """This rank's buffer ``name`` as ``[P, rows, W]`` bf16 (block i: the tokens of rank i)."""
        o = self._offset(name)
        return self.buf[o : o + self._tensor_bytes].view(torch.bfloat16).view(self.P, self.rows, self.W)

    def block_ptrs(self, name: str) -> list[int]:
        """Address of block ``rank`` of buffer ``name`` on every rank: where this rank's q/k/v column block j goes
        (rank j's heads), and where its out projection reads rank j's attention output for its own tokens."""
        o = self._offset(name) + self.rank * self.rows * self.W * 2
        return [b + o for b in self.base]

    def step(self) -> None:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF

    def copy_out(self, name: str, packed: Tensor) -> None:
        """Moves ``packed`` (``[P, rows, W]``, block j for rank j) into every rank's receive buffer ``name`` at this
        rank's slot, on the copy stream, after the work queued so far on the current stream (the GEMM that wrote it).
        ``join_copies`` makes the current stream wait for these copies."""
        compute = torch.cuda.current_stream(self.device)
        self.copy_stream.wait_stream(compute)
        dst = (ctypes.c_void_p * self.P)(*self.block_ptrs(name))
        src = (ctypes.c_void_p * self.P)(*[packed[j].data_ptr() for j in range(self.P)])
        nbytes = (ctypes.c_size_t * self.P)(*([self.rows * self.W * 2] * self.P))
        stream = ctypes.c_void_p(self.copy_stream.cuda_stream)
        self._lib.check(self._lib.lib().convrot_copy_blocks(dst, src, nbytes, self.P, stream), "convrot_copy_blocks")
        packed.record_stream(self.copy_stream)  # not recycled by the allocator before the copies have read it

    def pull_rows(self, name: str, r0: int, r1: int):
        """Rows [r0, r1) of block ``rank`` of every other rank's buffer ``name`` (this rank's tokens, their heads)
        into the staging buffer, by the copy engines on the copy stream, after the work queued so far on the current
        stream.  Returns an event recorded after the copies and the P row addresses to read: the staging rows for
        the other ranks, this rank's own buffer for itself."""
        self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        row_bytes = self.W * 2
        src_all = [b + r0 * row_bytes for b in self.block_ptrs(name)]
        others = [j for j in range(self.P) if j != self.rank]
        dst = (ctypes.c_void_p * len(others))(*[self.pull_stage[j, r0].data_ptr() for j in others])
        src = (ctypes.c_void_p * len(others))(*[src_all[j] for j in others])
        nbytes = (ctypes.c_size_t * len(others))(*([(r1 - r0) * row_bytes] * len(others)))
        stream = ctypes.c_void_p(self.copy_stream.cuda_stream)
        self._lib.check(self._lib.lib().convrot_copy_blocks(dst, src, nbytes, len(others), stream),
                        "convrot_copy_blocks")
        done = torch.cuda.Event()
        done.record(self.copy_stream)
        ptrs = [src_all[j] if j == self.rank else self.pull_stage[j, r0].data_ptr() for j in range(self.P)]
        return done, ptrs

    def join_copies(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self.copy_stream)

    def signal(self, phase: int) -> None:
        slots = (ctypes.c_void_p * self.P)(*[b + 4 * (8 * phase + self.rank) for b in self.base])
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        self._lib.check(self._lib.lib().convrot_peer_signal(slots, self.P, self.epoch, stream), "convrot_peer_signal")
        self.kernel_launches += 1

    def wait(self, phase: int) -> None:
        flags = ctypes.c_void_p(self.buf.data_ptr() + 4 * 8 * phase)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        self._lib.check(self._lib.lib().convrot_peer_wait(flags, self.P, self.epoch, stream), "convrot_peer_wait")
        self.kernel_launches += 1

    def _unmap(self) -> None:
        L = self._lib.lib()
        for mapped in self._opened:
            L.convrot_ipc_close(ctypes.c_void_p(mapped))
        self._opened = []

    def close(self) -> None:
        """Unmaps the other ranks' buffers; every rank calls it, after its last use of the exchange."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # nobody touches a peer's buffer any more
        self._unmap()
        dist.barrier(group=self.group)  # nobody maps this rank's buffer any more: it may be freed
        self.base = []
        self.buf = None


def attention_block_peer(x: Tensor, to_q, to_k, to_v, to_out, exchange: PeerExchange, attention=None) -> Tensor:
    """``attention_block_linears`` with the exchange fused into the kernels over peer memory (see PeerExchange)."""
    ex = exchange
    m = x.reshape(-1, x.shape[-1]).shape[0]
    if m != ex.rows or to_q.out_features != ex.width:
        raise ValueError(f"exchange is for {ex.rows} x {ex.width}, got {m} x {to_q.out_features}")
    P, d = ex.P, ex.width // ex.heads
    ex.step()
    for name, layer in zip("qkv", (to_q, to_k, to_v)):
        if name in ex.copy_names:
            ex.copy_out(name, layer(x, out_chunks=P))  # local send layout, then the copy engines
        else:
            layer.forward_scatter(x, ex.block_ptrs(name), ex.W)
    if ex.copy_names:
        ex.join_copies()
    ex.signal(ex.ARRIVED)
    ex.wait(ex.ARRIVED)
    if attention is None:
        source = "v"  # identity attention: the output is v as received
    else:
        qh, kh, vh = (ex.recv(n).view(P * m, ex.heads // P, d) for n in "qkv")
        ex.recv("out").copy_(attention(qh, kh, vh).reshape(P, m, ex.W))
        source = "out"
    ex.signal(ex.READY)
    ex.wait(ex.READY)
    if ex.pull_chunks <= 0:
        return to_out.forward_gather(ex.block_ptrs(source), m, ex.W, x.device)
    # The copy engines pull chunk c's rows from the other ranks while the compute stream runs the out projection of
    # chunk c - 1 on local memory (the chunk_block pattern, transformer.py:371-380); each chunk's output lands in
    # its rows of y.  The compute stream waits for every pull before the step ends, so ARRIVED of the next step
    # still follows this step's reads of the other ranks' buffers.
    n = ex.pull_chunks
    bounds = [(m * c // n, m * (c + 1) // n) for c in range(n)]
    pulls = [ex.pull_rows(source, r0, r1) for r0, r1 in bounds]
    y = torch.empty(m, to_out.out_features, dtype=torch.bfloat16, device=x.device)
    compute = torch.cuda.current_stream(x.device)
    for (r0, r1), (done, ptrs) in zip(bounds, pulls):
        compute.wait_event(done)
        to_out.forward_gather(ptrs, r1 - r0, ex.W, x.device, out=y[r0:r1])
    return y


def _packed_capable(x: Tensor, layers) -> bool:
    return x.is_cuda and all(hasattr(layer, "forward_packed") for layer in layers)


def attention_block_linears(x: Tensor, to_q, to_k, to_v, to_out, heads: int, attention=None, group=None,
                            exchange: PeerExchange | None = None) -> Tensor:
    """One attention block's linears on this rank's tokens: q/k/v (sharing one quantisation -- and one low-rank
    projection, see ``int8.share_lowrank`` -- when the layers have ``keep_input``), the seq->head all-to-all,
    ``attention`` (identity -> v when None), head->seq, and ``to_out``.

    With convrot layers on CUDA and more than one rank:

    * given an ``exchange`` (``PeerExchange``), the all-to-alls are fused into the kernels over peer memory;
    * otherwise the q/k/v GEMMs write their outputs straight into the NCCL all-to-all send layout
      ``[P, M/P, heads/P * D]`` and ``to_out`` reads the receive layout in place, so no pack or unpack copy surrounds
      the collectives; each q/k/v all-to-all is issued as soon as its GEMM is queued and overlaps the next GEMM."""
    P = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
    if exchange is not None and P > 1:
        return attention_block_peer(x, to_q, to_k, to_v, to_out, exchange, attention)
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
