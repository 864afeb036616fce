"""Multi-GPU partitioning of the attention path: one process per GPU.

Batch sharding (the primary mode): the sequences of a batch are split into G
shards of about equal total KV length (longest first, each to the shard with
the least work so far). Every GPU keeps the KV of its own sequences, so a step
needs no collective at all.

Head sharding (the variant): every GPU holds all sequences but only a
contiguous range of n_kv / G KV heads, with the query heads of those groups
(GQA keeps a group on one GPU). Each GPU computes out[B, Hq/G, hd] for its
heads; one all-gather per layer (NCCL over NVLink on GPUs, gloo on CPU) puts
out[B, Hq, hd] together on every rank. The q/k/v a rank passes in are its own
head slices, as a column-parallel projection produces them.

A rank that fails before a collective makes the others' collective fail with
the process group's timeout (an exception, not a hang); callers open the group
with a short timeout for that reason.
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


class HeadShardedAttn:
    """An ndattn.Attn over this rank's KV heads, with decode/prefill whose output
    is gathered over all ranks. Geometry arguments are those of the whole
    model; q/k/v/gate passed in are this rank's head slices."""

    def __init__(self, rank: int, world: int, n_heads: int, n_kv_heads: int, group=None, **kw):
        self.kv0, self.kv1, self.q0, self.q1 = head_range(n_heads, n_kv_heads, world, rank)
        self.group = group
        self.attn = ndattn.Attn(n_heads=self.q1 - self.q0, n_kv_heads=self.kv1 - self.kv0, **kw)

    def decode(self, layer, n, q, k, v, out_local, gate=None, seq_ids=None):
        """Local decode into out_local [n, Hloc * vd]; returns the gathered
        [n, Hq * vd]. The all-gather runs on the handle's stream, after the
        kernel."""
        import torch

        self.attn.decode(layer, n, q, k, v, out_local, gate=gate, seq_ids=seq_ids)
        with torch.cuda.stream(torch.cuda.ExternalStream(self.attn.stream)):
            return gather_heads(out_local, self.group)

    def close(self):
        self.attn.close()
