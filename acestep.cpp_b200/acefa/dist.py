"""Head-sharded attention across the GPUs of one node (one process per GPU).

acestep.cpp runs every module on one device (src/backend.h:97-101).  For long
DiT sequences (S up to 7500, docs/ARCHITECTURE.md:947-950) the attention of one
layer splits cleanly by K/V head group: rank r owns K/V heads
[r*Hkv/N, (r+1)*Hkv/N) and the Q heads that read them, computes its part of
ggml_flash_attn_ext with the local kernel, and one all-gather of the per-rank
output shards restores the full [D, Hq, S, B] result.  No other exchange is
needed: the mask is shared by all heads and every rank holds its own Q/K/V
head shard (in a sharded DiT the projections are sharded the same way).

Two ways to assemble the full output on every rank:

* ShardedOp: the kernel writes a contiguous [B, S, Hq/N, D] shard, an NCCL
  all_gather_into_tensor gives [N, B, S, Hq/N, D] and one permute gives
  [B, S, Hq, D] (two extra passes over the output in HBM).
* MirroredShardedOp: every rank maps every peer's full [B, S, Hq, D] output
  buffer (CUDA IPC through the C ABI) and the kernel's output stage stores
  each row into its head slice of all of them -- this GPU's buffer and, over
  NVLink, the peers' -- while later tiles are still computing.  A one-element
  NCCL all-reduce after the kernel is the completion barrier.  No gather, no
  permute, no extra HBM pass.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    hq0: int  # first Q head of this rank
    hq1: int  # one past the last
    hk0: int  # first K/V head
    hk1: int


def head_shard(Hq: int, Hkv: int, world: int, rank: int) -> HeadShard:
    """K/V head groups split evenly; each rank keeps whole GQA groups."""
    if Hkv % world != 0:
        raise ValueError(f"{Hkv} K/V heads do not split over {world} ranks")
    if Hq % Hkv != 0:
        raise ValueError("Hq must be a multiple of Hkv")
    G = Hq // Hkv
    per = Hkv // world
    hk0, hk1 = rank * per, (rank + 1) * per
    return HeadShard(rank, world, hk0 * G, hk1 * G, hk0, hk1)


def gather_heads(shard_out: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather [B, S, Hs, D] shards into [B, S, world*Hs, D]."""
    shard_out = shard_out.contiguous()
    B, S, Hs, D = shard_out.shape
    if world == 1:
        return shard_out
    gathered = torch.empty((world,) + tuple(shard_out.shape), dtype=shard_out.dtype, device=shard_out.device)
    backend = dist.get_backend(group)
    if backend == "nccl":
        dist.all_gather_into_tensor(gathered, shard_out, group=group)
    else:  # gloo: list form
        dist.all_gather(list(gathered.unbind(0)), shard_out, group=group)
    return gathered.permute(1, 2, 0, 3, 4).reshape(B, S, world * Hs, D)


def sharded_attention(q_shard: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                      mask: torch.Tensor | None, world: int, group=None,
                      compute: Callable | None = None, **op_kwargs) -> torch.Tensor:
    """This rank's heads through `compute` (default: the acefa kernel), then the
    all-gather.  q_shard (B, Hs, S, D) f32; k/v_shard (B, Hks, S_kv, D);
    returns the full (B, S, Hq, D) output on every rank."""
    if compute is None:
        import acefa

        out = acefa.flash_attn_ext(q_shard, k_shard, v_shard, mask, **op_kwargs)
    else:
        out = compute(q_shard, k_shard, v_shard, mask, **op_kwargs)
    return gather_heads(out, world, group)


class ShardedOp:
    """A captured-graph-friendly sharded node: the local op and the gather
    buffers are allocated once; __call__ launches the kernel and the NCCL
    all-gather on the current stream."""

    def __init__(self, q_shard, k_shard, v_shard, mask, world, group=None, **op_kwargs):
        import acefa

        self.world, self.group = world, group
        self.op = acefa.Op(q_shard, k_shard, v_shard, mask=mask, **op_kwargs)
        B, S, Hs, D = self.op.out.shape
        self.gathered = torch.empty((world, B, S, Hs, D), dtype=torch.float32, device=q_shard.device)
        self.out = torch.empty((B, S, world * Hs, D), dtype=torch.float32, device=q_shard.device)

    def __call__(self, stream=None):
        self.op(stream)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.op.out, group=self.group)
            self.out.copy_(self.gathered.permute(1, 2, 0, 3, 4).reshape(self.out.shape))
        else:
            self.out.copy_(self.op.out)
        return self.out


class MirroredShardedOp:
    """Head-sharded attention whose kernel stores the output straight into
    every rank's full (B, S, Hq, D) buffer (plain P2P stores over NVLink from
    the kernel's output stage; acefa_flash_attn_ext_mirrored).

    Collective at construction (handle exchange) and at every call (the
    completion barrier): all ranks construct and call it in the same order.
    The returned buffer is overwritten by the peers' next call, so its readers
    on this rank must finish before any rank starts the next call (true when
    other collectives separate consecutive attention layers)."""

    def __init__(self, q_shard, k_shard, v_shard, mask, world, group=None, **op_kwargs):
        import acefa

        self.world, self.group = world, group
        self.rank = dist.get_rank(group) if world > 1 else 0
        B, Hs, S, D = q_shard.shape
        dev = q_shard.device
        self.out = torch.empty((B, S, world * Hs, D), dtype=torch.float32, device=dev)
        self.peers: list[int] = []
        if world > 1:
            mine = acefa.peer_export(self.out)
            handles = [None] * world
            dist.all_gather_object(handles, mine, group=group)
            self.peers = [acefa.peer_import(h, off) for r, (h, off) in enumerate(handles) if r != self.rank]
        slice_off = self.rank * Hs * D * self.out.element_size()
        view = self.out[:, :, self.rank * Hs:(self.rank + 1) * Hs, :]
        self.op = acefa.Op(q_shard, k_shard, v_shard, mask=mask, out=view,
                           mirrors=[a + slice_off for a in self.peers], **op_kwargs)
        self.flag = torch.zeros(1, dtype=torch.float32, device=dev)

    def __call__(self, stream=None):
        self.op(stream)
        if self.world > 1:
            dist.all_reduce(self.flag, group=self.group)  # every rank's rows have landed
        return self.out

    def close(self):
        """Unmap the peers' buffers (collective: no rank may still be writing)."""
        import acefa

        if self.peers:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            for a in self.peers:
                acefa.peer_release(a)
            self.peers = []
