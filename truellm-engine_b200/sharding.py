"""Multi-GPU layouts of the paged KIVI decode path (one process per GPU).

The path shards three ways (no collective inside a decode step except where
the work of one sequence is split by tokens):

* by sequence -- each rank owns whole sequences.  `balance_sequences` assigns
  them by greedy token balancing (longest first, to the least-loaded rank),
  the continuous-batching layout;
* by kv head -- each rank owns `Hkv / N` kv heads and their q-head group
  (`head_shard`); every rank sees every sequence, outputs are disjoint head
  slices of `[B, Hq, D]`;
* by tokens of one sequence (long context) -- each rank owns a contiguous
  range of the 512-token quantised splits (`split_ranges`; the fp16 residual
  window belongs to the last rank).  Each rank computes its range and reduces
  it to one unnormalised partial per q head; the kernel that reduces it
  stores it straight into every rank's exchange buffer over NVLink (CUDA IPC
  mappings, `PeerExchange`) and raises a flag, and one more kernel per rank
  waits for all flags and merges the world slots with the log-sum-exp rule of
  paged_attention_v2.cu:132-170 (`tkv_exchange_decode_range`,
  `tkv_exchange_merge`).  The exchange is `(m, l)` plus `o[D]` fp32 per q head
  per rank: kilobytes per step.  The same layout over NCCL (all-gather of the
  one-slot partials of `tkv_paged_decode_range`, then `tkv_merge_partials`)
  remains as `exchange="nccl"`.

The functions here are plain host logic over torch tensors and
`torch.distributed`; `TokenSplitDecoder` and `PeerExchange` call the CUDA
entry points and therefore need the library and CUDA tensors (the group of a
`PeerExchange` only swaps IPC handles, so gloo serves), while `gather_slots`
and the planning helpers also run on CPU tensors with the gloo backend.
"""
from __future__ import annotations

import importlib
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

SPLIT_TOKENS = 512  # tokens per quantised split (TKV_SPLIT_TOKENS)


# ---------------------------------------------------------------------------
# planning
# ---------------------------------------------------------------------------
def balance_sequences(lengths: Sequence[int], world: int) -> List[np.ndarray]:
    """Greedy token balancing: sequences in decreasing length (ties: lower
    index first) go to the rank with the fewest tokens so far (ties: lower
    rank).  Returns each rank's sequence indices in increasing order."""
    lengths = np.asarray(lengths, np.int64)
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    owned: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owned[r].append(i)
        load[r] += int(lengths[i])
    return [np.asarray(sorted(o), np.int64) for o in owned]


def split_ranges(n_splits: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous quantised-split ranges [lo, hi) per rank covering
    [0, n_splits): the first n_splits % world ranks get one split more."""
    if world < 1 or n_splits < 0:
        raise ValueError("bad split plan")
    base, extra = divmod(n_splits, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def head_shard(n_kv_heads: int, n_q_heads: int, world: int, rank: int) -> Tuple[range, range]:
    """kv heads and q heads owned by `rank` when kv heads are split evenly."""
    if n_kv_heads % world or n_q_heads % n_kv_heads:
        raise ValueError(f"{n_kv_heads} kv heads do not split over {world} ranks")
    per = n_kv_heads // world
    grp = n_q_heads // n_kv_heads
    kv = range(rank * per, (rank + 1) * per)
    return kv, range(kv.start * grp, kv.stop * grp)


def quantized_splits(max_context_len: int, residual: int, group: int) -> int:
    """Quantised splits a decode over contexts up to max_context_len needs."""
    x = max_context_len - residual
    nq = group * (x // group) if x > 0 else 0
    return (nq + SPLIT_TOKENS - 1) // SPLIT_TOKENS


# ---------------------------------------------------------------------------
# exchange
# ---------------------------------------------------------------------------
def gather_slots(part_ml: torch.Tensor, part_o: torch.Tensor,
                 group: Optional[dist.ProcessGroup] = None,
                 out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gathers every rank's slot block ([S_local, B, Hq, 2] and
    [S_local, B, Hq, D], the same S_local on all ranks) into
    [world * S_local, ...] in rank order (into `out` when given)."""
    world = dist.get_world_size(group)
    if out is None:
        out = (torch.empty((world * part_ml.shape[0],) + tuple(part_ml.shape[1:]),
                           dtype=part_ml.dtype, device=part_ml.device),
               torch.empty((world * part_o.shape[0],) + tuple(part_o.shape[1:]),
                           dtype=part_o.dtype, device=part_o.device))
    ml, o = out
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(ml, part_ml.contiguous(), group=group)
        dist.all_gather_into_tensor(o, part_o.contiguous(), group=group)
    else:
        dist.all_gather(list(ml.chunk(world)), part_ml.contiguous(), group=group)
        dist.all_gather(list(o.chunk(world)), part_o.contiguous(), group=group)
    return ml, o


class PeerExchange:
    """One exchange buffer per rank (`tkv_device_alloc`), mapped into every
    other rank of `group` over CUDA IPC: the `tkv_exchange_t` of this rank.
    The group only carries the IPC handles (any backend).  `close()` unmaps
    and frees (collective)."""

    def __init__(self, batch: int, n_q_heads: int, head_dim: int,
                 group: Optional[dist.ProcessGroup] = None):
        self.ops = importlib.import_module("truellm-engine_b200.ops")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        nbytes = self.ops.exchange_buffer_bytes(self.world, batch, n_q_heads, head_dim)
        if nbytes == 0:
            raise ValueError(f"no exchange for world {self.world}")
        self.own = self.ops.DeviceBuffer(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, self.ops.ipc_handle(self.own.ptr), group=group)
        self.opened = {r: self.ops.ipc_open(h) for r, h in enumerate(handles) if r != self.rank}
        buffers = [self.own.ptr if r == self.rank else self.opened[r] for r in range(self.world)]
        self.ex = self.ops.exchange_struct(self.world, self.rank, buffers)
        dist.barrier(group=group)  # every mapping exists before any rank publishes

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still stores into a buffer
        for p in self.opened.values():
            self.ops.ipc_close(p)
        self.opened = {}
        dist.barrier(group=self.group)
        self.own.close()


def local_exchanges(world: int, batch: int, n_q_heads: int, head_dim: int):
    """`world` exchanges whose buffers all live on the current GPU, for one
    process that plays every rank in turn (each rank's publish before any
    merge, so no kernel waits on one that has not run).  Returns (structs,
    buffers); close the buffers when done."""
    ops = importlib.import_module("truellm-engine_b200.ops")
    nbytes = ops.exchange_buffer_bytes(world, batch, n_q_heads, head_dim)
    bufs = [ops.DeviceBuffer(nbytes) for _ in range(world)]
    return [ops.exchange_struct(world, r, [b.ptr for b in bufs]) for r in range(world)], bufs


class TokenSplitDecoder:
    """Decode of sequences whose quantised splits are spread over the ranks
    of `group` by `split_ranges` (each rank's cache must hold the pages of its
    range; the last rank also holds the fp16 residual window).

    One rank: the one-call decode (`tkv_paged_decode`).
    exchange="peer" (default): every rank reduces its range to one partial
    per (sequence, q head) and stores it into every rank's exchange buffer
    over NVLink (`tkv_exchange_decode_range`), then merges the world slots
    once all have arrived (`tkv_exchange_merge`): two launches per step per
    rank, no NCCL.  exchange="nccl": the one-slot partials of
    `tkv_paged_decode_range` are all-gathered (`(2 + D) * 4` bytes per q head
    per rank) and merged by `tkv_merge_partials`.  Buffers are allocated once
    per (batch, heads, context) shape; `close()` releases the peer mappings.
    """

    def __init__(self, batch: int, n_q_heads: int, head_dim: int, max_context_len: int,
                 residual: int, group_size: int, device,
                 group: Optional[dist.ProcessGroup] = None, exchange: str = "peer"):
        self.ops = importlib.import_module("truellm-engine_b200.ops")
        if exchange not in ("peer", "nccl"):
            raise ValueError(f"exchange must be 'peer' or 'nccl', not {exchange!r}")
        self.exchange = exchange
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        n = quantized_splits(max_context_len, residual, group_size)
        self.lo, self.hi = split_ranges(n, self.world)[self.rank]
        self.last = self.rank == self.world - 1
        self.active = self.hi > self.lo or self.last
        # one GPU: no split to exchange, the one-call decode
        self.single = self.world == 1
        self.max_context_len = max_context_len
        self.peer = (PeerExchange(batch, n_q_heads, head_dim, group)
                     if exchange == "peer" and not self.single else None)
        shape = (1, batch, n_q_heads)
        self.part_ml = torch.empty(shape + (2,), dtype=torch.float32, device=device)
        self.part_o = torch.zeros(shape + (head_dim,), dtype=torch.float32, device=device)
        self.part_ml[..., 0] = float("-inf")  # a rank without splits contributes nothing
        self.part_ml[..., 1] = 0.0
        self.ws = torch.zeros(max(16, self.ops.decode_range_workspace_bytes(
            batch, n_q_heads, head_dim, self.lo, self.hi),
            self.ops.decode_workspace_bytes(batch, n_q_heads, head_dim, max_context_len)),
            dtype=torch.uint8, device=device)
        self.all_ml = torch.empty((self.world,) + shape[1:] + (2,), dtype=torch.float32,
                                  device=device)
        self.all_o = torch.empty((self.world,) + shape[1:] + (head_dim,), dtype=torch.float32,
                                 device=device)

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def __call__(self, cache, q: torch.Tensor, block_tables: torch.Tensor,
                 seq_lens: torch.Tensor, out: torch.Tensor, scale: Optional[float] = None,
                 err: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        if self.single:
            return self.ops.paged_decode(cache, q, block_tables, seq_lens, self.max_context_len,
                                         scale=scale, out=out, workspace=self.ws, err=err,
                                         stream=stream)
        if self.peer is not None:
            self.ops.exchange_decode_range(
                cache, q, block_tables, seq_lens, self.lo, self.hi, self.last, self.peer.ex,
                self.ws, scale=scale, err=err, stream=stream)
            return self.ops.exchange_merge(self.peer.ex, out, err=err, stream=stream)
        if self.active:
            self.ops.paged_decode_range(
                cache, q, block_tables, seq_lens, self.lo, self.hi, self.last,
                self.part_ml[0], self.part_o[0], self.ws, scale=scale, err=err, stream=stream)
        gather_slots(self.part_ml, self.part_o, self.group, out=(self.all_ml, self.all_o))
        return self.ops.merge_partials(self.all_ml, self.all_o, out, stream=stream)

    def capture(self, cache, q: torch.Tensor, block_tables: torch.Tensor,
                seq_lens: torch.Tensor, out: torch.Tensor, scale: Optional[float] = None,
                err: Optional[torch.Tensor] = None) -> "torch.cuda.CUDAGraph":
        """Records one call (range decode, reduce, all-gather, merge) over these
        fixed buffers in a CUDA graph; `graph.replay()` reruns it with one host
        launch.  Every rank of the group must capture (the graph holds the
        collectives); release the graph before destroying the group."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # first call eagerly: communicator set-up
            self(cache, q, block_tables, seq_lens, out, scale=scale, err=err,
                 stream=torch.cuda.current_stream())
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self(cache, q, block_tables, seq_lens, out, scale=scale, err=err,
                 stream=torch.cuda.current_stream())
        return graph

