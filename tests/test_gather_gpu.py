"""Head-sharded decode (nd_attn_decode_gather) on the GPU, through the C ABI.

- One rank (world 1) on one GPU: the attention kernels store the output rows
  into the gather slot, the launch's last CTA publishes its flag, and the wait
  kernel copies the slot out; several calls in a row alternate the two slots
  and counters. The output equals the plain decode's bit for bit (the same
  kernels and plans), on the balanced 16-bit kernel and on the exact-grid
  kernel (int8 caches with two KV heads).
- Two ranks on two GPUs (skipped with fewer): each rank holds half the KV
  heads, every rank's output holds all heads, within the parity tolerance of a
  handle that holds all heads on one GPU. Then rank 1 skips a call: rank 0's
  bounded wait expires and nd_attn_sync reports ND_ATTN_ERR_TIMEOUT.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

import ndattn
from harness import TOL, rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _fill(a, ctx, seed, n_layers, width_k, width_v, kv):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    for layer in range(n_layers):
        for s, n in enumerate(ctx):
            k = torch.randn((n, width_k), generator=g, device="cuda") * 0.5
            v = torch.randn((n, width_v), generator=g, device="cuda") * 0.5
            torch.cuda.synchronize()
            if kv == "i8":
                hk = a.cfg.n_kv_heads
                ks = (k.view(n, hk, -1).abs().amax(2) / 127).contiguous()
                vs = (v.view(n, hk, -1).abs().amax(2) / 127).contiguous()
                k8 = torch.round(k.view(n, hk, -1) / ks[..., None]).clamp(-127, 127).to(torch.int8).view(n, -1)
                v8 = torch.round(v.view(n, hk, -1) / vs[..., None]).clamp(-127, 127).to(torch.int8).view(n, -1)
                a.write_cache(layer, s, 0, n, k8.contiguous(), v8.contiguous(), ks, vs)
            else:
                a.write_cache(layer, s, 0, n, k.half().contiguous(), v.half().contiguous())
        torch.cuda.synchronize()
    for s, n in enumerate(ctx):
        a.set_state(s, n, 0)


@pytest.mark.parametrize("kv,H,HKV", [("f16", 8, 8), ("i8", 8, 2)])
def test_gathered_decode_one_rank_matches_plain_decode(kv, H, HKV):
    import torch
    ctx = [300, 1999, 64, 1024, 777]
    B, L, D = len(ctx), 2, 64
    act = "f16" if kv == "f16" else "f32"
    tdt = torch.float16 if act == "f16" else torch.float32
    mk = lambda: ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=HKV, window=2048 + 64, max_seqs=B,  # noqa: E731
                             kv_dtype=kv, act_dtype=act, out_dtype=act, max_pos=2048 + 64)
    plain, gath = mk(), mk()
    for a in (plain, gath):
        _fill(a, ctx, 21, L, HKV * D, HKV * D, kv)
    rec = gath.gather_init(0, 1)
    ndattn.gather_check(rec, 1, 0)
    gath.gather_attach(rec)
    g = torch.Generator(device="cuda")
    g.manual_seed(22)
    launches0 = gath.launches
    for step in range(3):
        for layer in range(L):
            q = torch.randn((B, H * D), generator=g, device="cuda").to(tdt)
            k = (torch.randn((B, HKV * D), generator=g, device="cuda") * 0.5).to(tdt)
            v = (torch.randn((B, HKV * D), generator=g, device="cuda") * 0.5).to(tdt)
            gt = torch.randn((B, H * D), generator=g, device="cuda").to(tdt)
            o1 = torch.zeros((B, H * D), dtype=tdt, device="cuda")
            o2 = torch.full((B, H * D), float("nan"), dtype=tdt, device="cuda")
            plain.decode(layer, B, q, k, v, o1, gate=gt)
            gath.decode_gather(layer, B, q, k, v, o2, gate=gt)
            plain.sync()
            gath.sync()
            assert torch.equal(o1.view(torch.int16 if act == "f16" else torch.int32),
                               o2.view(torch.int16 if act == "f16" else torch.int32)), (step, layer)
        plain.advance(B)
        gath.advance(B)
    # per call the attend launch and the wait-and-copy, per step the position advance
    assert gath.launches - launches0 == 3 * (L * 2 + 1)
    for layer in range(L):
        for s in range(B):
            kp, vp, _, _ = plain.read_cache(layer, s, 0, ctx[s] + 3)
            kg, vg, _, _ = gath.read_cache(layer, s, 0, ctx[s] + 3)
            assert np.array_equal(kp.view(np.uint8), kg.view(np.uint8))
            assert np.array_equal(vp.view(np.uint8), vg.view(np.uint8))
    plain.close()
    gath.close()


def test_gathered_decode_refused_before_attach():
    import torch
    a = ndattn.Attn(n_heads=8, n_kv_heads=8, window=128, max_seqs=2, kv_dtype="f16", act_dtype="f16")
    z = torch.zeros((2, 512), dtype=torch.float16, device="cuda")
    with pytest.raises(ndattn.NdAttnError) as e:
        a.decode_gather(0, 2, z, z, z, z)
    assert e.value.code == ndattn.ERR_ARG
    a.gather_init(0, 1)
    with pytest.raises(ndattn.NdAttnError):
        a.gather_init(0, 1)                    # once per handle
    a.close()


# ------------------------------------------------------------------ two GPUs
def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_rank_worker(rank, world, port, result_path):
    sys.path[:0] = [HERE, os.path.join(HERE, "..", "oracle"), os.path.join(HERE, "..", "esp32-needle-3_b200")]
    import torch
    import torch.distributed as dist

    import ndattn as N
    import ndshard as S
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    msgs = []
    for kv, H, HKV in (("f16", 8, 8), ("i8", 16, 8)):
        ctx = [256, 2048, 1000, 513, 64, 1500]
        B, L, D, W = len(ctx), 2, 64, 2048 + 64
        act = "f16" if kv == "f16" else "f32"
        tdt = torch.float16 if act == "f16" else torch.float32
        sh = S.HeadShardedAttn(rank, world, H, HKV, n_layers=L, window=W, max_seqs=B, kv_dtype=kv, act_dtype=act,
                               out_dtype=act, max_pos=W, device=rank)
        full = N.Attn(n_layers=L, n_heads=H, n_kv_heads=HKV, window=W, max_seqs=B, kv_dtype=kv, act_dtype=act,
                      out_dtype=act, max_pos=W, device=rank)
        _fill(full, ctx, 31, L, HKV * D, HKV * D, kv)
        # The sharded handle's caches: this rank's head columns of the full one.
        for layer in range(L):
            for s, n in enumerate(ctx):
                k, v, ks, vs = full.read_cache(layer, s, 0, n)
                c0, c1 = sh.kv0 * D, sh.kv1 * D
                kk = torch.from_numpy(np.ascontiguousarray(k[:, c0:c1])).cuda()
                vv = torch.from_numpy(np.ascontiguousarray(v[:, c0:c1])).cuda()
                sk = sv = None
                if kv == "i8":
                    sk = torch.from_numpy(np.ascontiguousarray(ks[:, sh.kv0:sh.kv1])).cuda()
                    sv = torch.from_numpy(np.ascontiguousarray(vs[:, sh.kv0:sh.kv1])).cuda()
                sh.attn.write_cache(layer, s, 0, n, kk, vv, sk, sv)
                torch.cuda.synchronize()
        for s, n in enumerate(ctx):
            sh.attn.set_state(s, n, 0)
        g = torch.Generator(device="cuda")
        g.manual_seed(32)                      # the same full-head inputs on both ranks
        worst = 0.0
        for step in range(3):
            for layer in range(L):
                q = torch.randn((B, H, D), generator=g, device="cuda").to(tdt)
                k = (torch.randn((B, HKV, D), generator=g, device="cuda") * 0.5).to(tdt)
                v = (torch.randn((B, HKV, D), generator=g, device="cuda") * 0.5).to(tdt)
                o_full = torch.zeros((B, H * D), dtype=tdt, device="cuda")
                o_sh = torch.full((B, H * D), float("nan"), dtype=tdt, device="cuda")
                full.decode(layer, B, q.reshape(B, -1), k.reshape(B, -1), v.reshape(B, -1), o_full)
                sh.decode(layer, B, q[:, sh.q0:sh.q1].contiguous().reshape(B, -1),
                          k[:, sh.kv0:sh.kv1].contiguous().reshape(B, -1),
                          v[:, sh.kv0:sh.kv1].contiguous().reshape(B, -1), o_sh)
                full.sync()
                sh.attn.sync()
                worst = max(worst, rel_err(o_sh.float().cpu().numpy(), o_full.float().cpu().numpy()))
            full.advance(B)
            sh.attn.advance(B)
        msgs.append(f"{kv} {worst:.3e}")
        full.close()
        if kv == "i8":
            # Rank 1 leaves out one gathered call: rank 0's wait for it expires.
            if rank == 0:
                z = torch.zeros((B, (sh.q1 - sh.q0) * D), dtype=tdt, device="cuda")
                zk = torch.zeros((B, (sh.kv1 - sh.kv0) * D), dtype=tdt, device="cuda")
                o = torch.zeros((B, H * D), dtype=tdt, device="cuda")
                sh.decode(0, B, z, zk, zk, o)
                try:
                    sh.attn.sync()
                    msgs.append("no timeout")
                except N.NdAttnError as e:
                    msgs.append(f"timeout {e.code}")
        sh.close()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("\n".join(msgs))
    dist.destroy_process_group()


def test_gathered_decode_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    path = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"ndgather_{os.getpid()}")
    mp.start_processes(_two_rank_worker, args=(2, _port(), path), nprocs=2, start_method="spawn")
    for r in range(2):
        with open(f"{path}.{r}") as f:
            lines = f.read().splitlines()
        os.remove(f"{path}.{r}")
        for ln in lines[:2]:
            kv, err = ln.split()
            assert float(err) <= TOL, (r, ln)
        if r == 0:
            assert lines[2] == f"timeout {ndattn.ERR_TIMEOUT}", lines
