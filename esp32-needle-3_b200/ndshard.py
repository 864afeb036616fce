"""Multi-GPU partitioning of the attention path: one process per GPU.

Batch sharding (the primary mode): the sequences of a batch are split into G
shards of about equal total KV length (longest first, each to the shard with
the least work so far). Every GPU keeps the KV of its own sequences, so a step
needs no collective at all.

Head sharding (the variant): every GPU holds all sequences but only a
contiguous range of n_kv / G KV heads, with the query heads of those groups
(GQA keeps a group on one GPU). The library's gathered decode
(nd_attn_decode_gather) computes the rank's heads and stores each output row
straight into every rank's gather buffer from inside the attention kernel
(peer stores over NVLink), so out[B, Hq, hd] is complete on every rank with no
collective library call and no permute. The process group only carries the
one-time exchange of the ranks' buffer records. The q/k/v a rank passes in are
its own head slices, as a column-parallel projection produces them.
gather_heads is the same gather written as a process-group all-gather: the
layout reference for the CPU tests.

A rank that fails before a gathered call makes the others' call end with
ND_ATTN_ERR_TIMEOUT (a bounded device wait), and a rank that fails before a
process-group collective makes the others' collective fail with the group's
timeout (an exception, not a hang); callers open the group with a short
timeout for that reason.
"""
from __future__ import annotations

import numpy as np

import ndattn


def balance_batch(ctx, n_shards: int) -> list[np.ndarray]:
    """Indices of the sequences of each shard: longest context first, each to
    the shard with the smallest total so far; every shard's indices sorted."""
    ctx = np.asarray(ctx, dtype=np.int64)
    if n_shards < 1:
        raise ValueError("n_shards must be >= 1")
    load = np.zeros(n_shards, dtype=np.int64)
    owner = np.empty(len(ctx), dtype=np.int64)
    for i in np.argsort(-ctx, kind="stable"):
        s = int(np.argmin(load))
        owner[i] = s
        load[s] += ctx[i]
    return [np.flatnonzero(owner == s) for s in range(n_shards)]


def head_range(n_heads: int, n_kv_heads: int, n_shards: int, rank: int) -> tuple[int, int, int, int]:
    """(kv0, kv1, q0, q1): the KV heads [kv0, kv1) and query heads [q0, q1)
    rank `rank` of `n_shards` owns. n_kv_heads must split evenly."""
    if n_kv_heads % n_shards or n_heads % n_kv_heads:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {n_shards} ranks")
    per = n_kv_heads // n_shards
    rep = n_heads // n_kv_heads
    kv0, kv1 = rank * per, (rank + 1) * per
    return kv0, kv1, kv0 * rep, kv1 * rep


def gather_heads(local_out, group=None):
    """[B, Hloc * hd] per rank -> [B, G * Hloc * hd] on every rank, rank r's
    heads at columns [r * Hloc * hd, (r + 1) * Hloc * hd)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    local_out = local_out.contiguous()
    b, cols = local_out.shape
    # Ranks concatenated along dim 0 (the form every backend accepts).
    buf = torch.empty((world * b, cols), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf, local_out, group=group)
    return buf.view(world, b, cols).permute(1, 0, 2).reshape(b, world * cols)


def exchange_records(record: bytes, group=None) -> bytes:
    """Every rank's gather record, concatenated in rank order: one all-gather
    over the process group (a uint8 tensor; on the GPU for NCCL groups)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
        else torch.device("cpu")
    mine = torch.tensor(list(record), dtype=torch.uint8, device=dev)
    allr = torch.empty(world * len(record), dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(allr, mine, group=group)
    return bytes(allr.cpu().numpy().tobytes())


class HeadShardedAttn:
    """An ndattn.Attn over this rank's KV heads whose decode gathers every
    rank's heads inside the library (nd_attn_decode_gather). Geometry arguments
    are those of the whole model; q/k/v/gate passed in are this rank's head
    slices. Construction and close() are collective over the group."""

    def __init__(self, rank: int, world: int, n_heads: int, n_kv_heads: int, group=None, **kw):
        import torch.distributed as dist

        self.kv0, self.kv1, self.q0, self.q1 = head_range(n_heads, n_kv_heads, world, rank)
        self.group, self.rank, self.world = group, rank, world
        self.attn = ndattn.Attn(n_heads=self.q1 - self.q0, n_kv_heads=self.kv1 - self.kv0, **kw)
        rec = self.attn.gather_init(rank, world)
        recs = exchange_records(rec, group) if world > 1 else rec
        ndattn.gather_check(recs, world, rank)
        self.attn.gather_attach(recs)
        if world > 1:
            dist.barrier(group)         # every rank mapped every buffer before the first call

    def decode(self, layer, n, q, k, v, out, gate=None, seq_ids=None):
        """Decode of this rank's heads; out [n, Hq * vd] receives every rank's
        heads (rank r's at columns [r * Hloc * vd, (r + 1) * Hloc * vd))."""
        self.attn.decode_gather(layer, n, q, k, v, out, gate=gate, seq_ids=seq_ids)

    def close(self):
        import torch.distributed as dist

        self.attn.sync()
        if self.world > 1:
            dist.barrier(self.group)    # no rank still writes into another's buffer
        self.attn.close()
