"""Multi-rank host logic on CPU (gloo, world size 2): the batch partition,
the head ranges, the head-sharded output gather, and a rank that fails before
the collective. Per-rank attention here is the oracle over the rank's heads
(the GPU path is exercised by bench.py under torchrun); what is under test is
the partition and gather code the GPU path uses."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

import ndoracle as O
import ndshard

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_balance_batch_partitions_and_balances():
    rng = np.random.default_rng(1)
    ctx = rng.integers(256, 2049, size=64)
    for g in (1, 2, 3, 4, 8):
        shards = ndshard.balance_batch(ctx, g)
        assert len(shards) == g
        allidx = np.sort(np.concatenate(shards))
        assert np.array_equal(allidx, np.arange(64))
        loads = [int(ctx[s].sum()) for s in shards]
        assert max(loads) - min(loads) <= int(ctx.max())   # greedy longest-first bound
    assert [len(s) for s in ndshard.balance_batch([5, 5], 4)] == [1, 1, 0, 0]


def test_head_ranges_cover_and_keep_groups():
    for n_heads, n_kv, g in ((8, 8, 8), (16, 4, 4), (16, 4, 2), (8, 8, 2)):
        got = [ndshard.head_range(n_heads, n_kv, g, r) for r in range(g)]
        assert [x[0] for x in got] == [r * n_kv // g for r in range(g)]
        assert got[-1][1] == n_kv and got[-1][3] == n_heads
        for kv0, kv1, q0, q1 in got:
            assert (q0, q1) == (kv0 * n_heads // n_kv, kv1 * n_heads // n_kv)
    with pytest.raises(ValueError):
        ndshard.head_range(8, 8, 3, 0)


def _session(seed, n_heads, n_kv, hd, ctx, q0, q1, kv0, kv1):
    """Oracle outputs [B, (q1-q0)*hd] of one decode step over the heads
    [q0, q1) / [kv0, kv1) of a seeded random session (same bytes on every rank)."""
    rng = np.random.default_rng(seed)
    B = len(ctx)
    W = max(ctx) + 8
    out = []
    for b in range(B):
        k = (rng.standard_normal((ctx[b], n_kv, hd)) * 0.5).astype(np.float16)
        v = (rng.standard_normal((ctx[b], n_kv, hd)) * 0.5).astype(np.float16)
        q = rng.standard_normal((n_heads, hd)).astype(np.float32)
        kn = (rng.standard_normal((n_kv, hd)) * 0.5).astype(np.float32)
        vn = (rng.standard_normal((n_kv, hd)) * 0.5).astype(np.float32)
        s = O.OracleSeq(1, q1 - q0, kv1 - kv0, hd, hd, W, O.F16, max_pos=W)
        s.k[0, :ctx[b]] = k[:, kv0:kv1].reshape(ctx[b], -1).view(np.uint16)
        s.v[0, :ctx[b]] = v[:, kv0:kv1].reshape(ctx[b], -1).view(np.uint16)
        s.pos = ctx[b]
        o = s.step(0, O.round_act(q[q0:q1].ravel(), O.F16), O.round_act(kn[kv0:kv1].ravel(), O.F16),
                   O.round_act(vn[kv0:kv1].ravel(), O.F16))
        out.append(np.asarray(o, dtype=np.float32).ravel())
    return np.stack(out)


def _gather_worker(rank, world, port, result_path):
    sys.path[:0] = [HERE, os.path.join(HERE, "..", "oracle"), os.path.join(HERE, "..", "esp32-needle-3_b200")]
    import torch
    import torch.distributed as dist

    import ndshard as S
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    n_heads, n_kv, hd, ctx = 16, 4, 64, [70, 200, 129]
    kv0, kv1, q0, q1 = S.head_range(n_heads, n_kv, world, rank)
    local = torch.from_numpy(_session(7, n_heads, n_kv, hd, ctx, q0, q1, kv0, kv1))
    full = S.gather_heads(local).numpy()
    if rank == 0:
        want = _session(7, n_heads, n_kv, hd, ctx, 0, n_heads, 0, n_kv)
        np.save(result_path, np.stack([full, want]))
    dist.destroy_process_group()


def test_head_sharded_gather_equals_all_heads():
    import torch.multiprocessing as mp
    path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"ndshard_{os.getpid()}.npy")
    mp.start_processes(_gather_worker, args=(2, _port(), path), nprocs=2, start_method="spawn")
    full, want = np.load(path)
    os.remove(path)
    assert full.shape == want.shape == (3, 16 * 64)
    assert np.array_equal(full, want)   # heads are independent: bit-identical


def _failing_worker(rank, world, port, result_path):
    sys.path[:0] = [HERE, os.path.join(HERE, "..", "esp32-needle-3_b200")]
    import torch
    import torch.distributed as dist

    import ndshard as S
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(3)   # dies between steps, before its collective
    try:
        S.gather_heads(torch.zeros((2, 8)))
        msg = "no error"
    except Exception as e:   # the survivor learns of it as an error, not a hang
        msg = "error: " + type(e).__name__
    with open(result_path, "w") as f:
        f.write(msg)
    os._exit(0)


def test_rank_failure_surfaces_as_error():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _port()
    path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"ndshard_fail_{os.getpid()}.txt")
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    with open(path) as f:
        msg = f.read()
    os.remove(path)
    assert msg.startswith("error"), msg


# ------------------------------------------------ gathered decode: record exchange
GATHER_MAGIC, GATHER_VERSION = 0x4147444E, 2


def _record(rank, world, gpu_id, row_words=256, max_tokens=64, out_dtype=2):
    """A gather record in the library's layout (the GatherBlob struct of
    nd_attn.cu: 6 u32, u64 slot bytes, 2 u32, GPU uuid, IPC handle, padding)
    with a fake IPC handle: what nd_attn_gather_init fills, for host-only
    checks of the exchange and of nd_attn_gather_check."""
    import struct
    slot = (max_tokens * row_words * 8 + 255) // 256 * 256
    head = struct.pack("<6IQ2I", GATHER_MAGIC, GATHER_VERSION, rank, world, max_tokens, row_words, slot, out_dtype,
                       0)
    return head + bytes([gpu_id] * 16) + bytes(64) + bytes(8)


def _records_worker(rank, world, port, result_path):
    sys.path[:0] = [HERE, os.path.join(HERE, "..", "esp32-needle-3_b200")]
    import torch.distributed as dist

    import ndattn
    import ndshard as S
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    recs = S.exchange_records(_record(rank, world, 0x10 + rank))
    try:
        ndattn.gather_check(recs, world, rank)
        msg = "ok"
    except ndattn.NdAttnError as e:
        msg = f"error {e.code}"
    if recs[rank * ndattn.GATHER_BLOB_BYTES:(rank + 1) * ndattn.GATHER_BLOB_BYTES] != _record(rank, world, 0x10 + rank):
        msg = "own record not at its rank's place"
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(msg)
    dist.destroy_process_group()


def test_gather_records_exchange_and_check():
    """The set-up of nd_attn_decode_gather on two gloo ranks: every rank's
    record ends up at its rank's place in every rank's array, and the
    library's host-side check accepts it; then the check refuses records out
    of rank order, two ranks on one GPU, unequal geometry and a world size
    that differs from the records'."""
    import torch.multiprocessing as mp

    import ndattn
    path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"ndshard_rec_{os.getpid()}")
    mp.start_processes(_records_worker, args=(2, _port(), path), nprocs=2, start_method="spawn")
    for r in range(2):
        with open(f"{path}.{r}") as f:
            assert f.read() == "ok"
        os.remove(f"{path}.{r}")
    ndattn.gather_check(_record(0, 2, 1) + _record(1, 2, 2), 2, 1)
    ndattn.gather_check(_record(0, 1, 1), 1, 0)
    bad = [_record(1, 2, 2) + _record(0, 2, 1),                     # out of rank order
           _record(0, 2, 1) + _record(1, 2, 1),                     # two ranks on one GPU
           _record(0, 2, 1) + _record(1, 2, 2, row_words=512),      # another geometry
           _record(0, 3, 1) + _record(1, 3, 2)]                     # records of a world of 3
    for b in bad:
        with pytest.raises(ndattn.NdAttnError) as e:
            ndattn.gather_check(b, 2, 0)
        assert e.value.code == ndattn.ERR_ARG
    with pytest.raises(ndattn.NdAttnError):
        ndattn.gather_check(_record(0, 2, 1) + _record(1, 2, 2), 2, 2)   # rank outside the world
