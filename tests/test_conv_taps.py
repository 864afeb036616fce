"""QKV short causal convolution (qkv_conv_taps = 3, tap_projection,
nd_model.c:2361-2379) ahead of the attention path on the GPU, against the
oracle, whose convolution and history rules are pinned to the reference's own
tap_projection and nd_model_snapshot (tests/test_oracle_pin.py).

One session per cache type walks every place the tap history matters:
- a first prefill from position 0 (the ramp of min(taps, pos+1) taps) with
  ragged lengths, 1 to 40 tokens;
- decode steps, then a second prefill that reads history across calls;
- snapshot, decode, rewind (the history goes back with the position);
- a saved prefix (image = live KV rows, then the snapshot's q/k/v histories,
  byte for byte) restored into another sequence;
- a reset (history cleared), then more tokens.
int8 runs the general kernels, f16 / bf16 at head dim 64 the tensor-core
prefill and the balanced decode, over MHA and query groups of two and four
rows. Outputs within TOL, caches bit-exact."""
import numpy as np
import pytest

import ndattn
import ndoracle as O
from harness import TOL, cache_bits, dev, oracle_cache, rel_err

pytestmark = pytest.mark.gpu

NAMES = {O.F32: "f32", O.F16: "f16", O.BF16: "bf16", O.I8: "i8"}


@pytest.mark.parametrize("kv_dt,act_dt,H,HKV", [(O.I8, O.F32, 8, 2), (O.F16, O.F16, 8, 2), (O.BF16, O.BF16, 8, 2),
                                                 (O.F16, O.F16, 4, 4), (O.BF16, O.BF16, 8, 4)])
def test_conv_taps_session(kv_dt, act_dt, H, HKV):
    import torch
    rng = np.random.default_rng(23 + kv_dt + H * HKV)
    L, HD, W, B, T = 2, 64, 256, 3, 3
    a = ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=HKV, window=W, max_seqs=B, kv_dtype=NAMES[kv_dt],
                    act_dtype=NAMES[act_dt], out_dtype="f32", qkv_conv_taps=T)
    seqs = [O.OracleSeq(L, H, HKV, HD, HD, W, kv_dt, taps=T, act_dtype=act_dt) for _ in range(B)]
    for l in range(L):
        ws = [(rng.standard_normal((T, d)) * 0.6).astype(np.float32) for d in (H * HD, HKV * HD, HKV * HD)]
        a.set_conv_taps(l, *ws)
        for s in seqs:
            s.set_conv_taps(l, *ws)
    worst = 0.0

    def call(lens, decode=False):
        nonlocal worst
        ids = [s for s in range(B) if lens[s]]
        n = sum(lens[s] for s in ids)
        q = (rng.standard_normal((n, H * HD)) * 0.5).astype(np.float32)
        k = (rng.standard_normal((n, HKV * HD)) * 0.5).astype(np.float32)
        v = (rng.standard_normal((n, HKV * HD)) * 0.5).astype(np.float32)
        for l in range(L):
            out = torch.zeros((n, H * HD), dtype=torch.float32, device="cuda")
            args = (dev(q, act_dt), dev(k, act_dt), dev(v, act_dt), out)
            if decode:
                a.decode(l, len(ids), *args, seq_ids=ids)
            else:
                a.prefill(l, [lens[s] for s in ids], *args, seq_ids=ids)
            a.sync()
            got = out.cpu().numpy()
            row = 0
            for s in ids:
                for t in range(lens[s]):
                    want = seqs[s].step(l, O.round_act(q[row], act_dt), O.round_act(k[row], act_dt),
                                        O.round_act(v[row], act_dt), off=t)
                    worst = max(worst, rel_err(got[row].reshape(H, HD), want))
                    row += 1
        a.advance(len(ids), seq_ids=ids, lens=[lens[s] for s in ids])
        for s in ids:
            seqs[s].advance(lens[s])

    call([5, 40, 1])
    for _ in range(3):
        call([1, 1, 1], decode=True)
    call([2, 3, 7])
    a.snapshot(1)
    seqs[1].snapshot()
    for _ in range(2):
        call([1, 1, 1], decode=True)
    a.rewind(1)
    seqs[1].rewind()
    call([0, 2, 0])
    a.snapshot(1)
    seqs[1].snapshot()
    pre = a.prefix_save(1)
    img, ppos, psink = pre.read()
    assert (ppos, psink) == (seqs[1].pos, seqs[1].n_sink)
    assert img.tobytes() == seqs[1].prefix_image()
    a.prefix_restore(2, pre)
    seqs[2].prefix_restore(seqs[1].prefix_save())
    for _ in range(2):
        call([1, 1, 1], decode=True)
    a.reset(0)
    seqs[0].reset()
    call([4, 1, 1])
    call([1, 1, 1], decode=True)
    assert worst <= TOL, worst
    for s, seq in enumerate(seqs):
        n = seq.pos
        for l in range(L):
            gk, gv, gks, gvs = a.read_cache(l, s, 0, n)
            ok, ov = oracle_cache(seq, l, kv_dt)
            assert np.array_equal(cache_bits(gk), cache_bits(ok[:n])), (s, l)
            assert np.array_equal(cache_bits(gv), cache_bits(ov[:n])), (s, l)
            if kv_dt == O.I8:
                assert np.array_equal(gks, seq.ks[l][:n]) and np.array_equal(gvs, seq.vs[l][:n])
    pre.free()
    a.close()


def test_conv_taps_allocation_free_decode_and_host_buffers():
    """The allocation-free decode and the host-buffer decode take the same
    convolution (their tap buffer is sized at open): both give the device
    entry point's bits, step after step."""
    import torch
    rng = np.random.default_rng(5)
    L, H, HD, W, B, T = 1, 4, 64, 128, 2, 3
    outs = {}
    steps = [[(rng.standard_normal((B, H * HD)) * 0.5).astype(np.float32) for _ in range(3)] for _ in range(4)]
    for form in ("device", "noalloc", "host"):
        a = ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=H, window=W, max_seqs=B, kv_dtype="f16",
                        act_dtype="f32", out_dtype="f32", qkv_conv_taps=T)
        wr = np.random.default_rng(9)
        a.set_conv_taps(0, *[(wr.standard_normal((T, H * HD)) * 0.6).astype(np.float32) for _ in range(3)])
        res = []
        for q, k, v in steps:
            if form == "host":
                out = np.zeros((B, H * HD), np.float32)
                a.decode_host(0, B, q, k, v, out)
                res.append(out)
            else:
                t = [torch.from_numpy(x).cuda() for x in (q, k, v)]
                o = torch.zeros((B, H * HD), device="cuda")
                if form == "device":
                    a.decode(0, B, *t, o)
                else:
                    a.decode_noalloc(0, B, *t, o)
                a.sync()
                res.append(o.cpu().numpy())
            a.advance(B)
        outs[form] = res
        a.close()
    for form in ("noalloc", "host"):
        for x, y in zip(outs["device"], outs[form]):
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), form


def test_conv_taps_geometry_checks():
    with pytest.raises(ndattn.NdAttnError) as e:
        ndattn.Attn(qkv_conv_taps=5)
    assert e.value.code == ndattn.ERR_GEOM
    a = ndattn.Attn()
    with pytest.raises(ndattn.NdAttnError) as e:
        a.set_conv_taps(0, np.zeros((1, 512)), np.zeros((1, 512)), np.zeros((1, 512)))
    assert e.value.code == ndattn.ERR_ARG
    a.close()
