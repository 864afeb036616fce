"""Parity of the TMA-staged decode kernel (16-bit caches, equal head dims 64 or
128, no position wrapping the ring) with the oracle.

Contexts are written straight into the cache at ragged lengths up to ~2k so
each sequence gets several splits whose starts are multiples of 64 rows, and
the tail of each split is a partial box. Unwritten rows and the rows of other
sequences hold NaN bit patterns: the kernel's boxes read them (a box is 64
rows, the context is not), so this checks that masked rows contribute nothing.
Bar: max|d| <= 1e-3 * max(1, |ref|) (harness.TOL); cache bytes bit-exact."""
import numpy as np
import pytest

import ndattn
import ndoracle as O
from harness import TOL, cache_bits, dev, oracle_cache, random_kv_rows, rel_err

pytestmark = pytest.mark.gpu


def _session(kv_dt, hd, rep, block_size, seed, ctx, steps=2, L=2):
    import torch
    rng = np.random.default_rng(seed)
    HKV = 2 if hd == 128 else 4
    H = HKV * rep
    W = 2304
    B = len(ctx)
    name = "f16" if kv_dt == O.F16 else "bf16"
    a = ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=HKV, qk_head_dim=hd, v_head_dim=hd, window=W, max_seqs=B,
                    kv_dtype=name, act_dtype=name, out_dtype="f32", block_size=block_size, max_pos=W)
    seqs = [O.OracleSeq(L, H, HKV, hd, hd, W, kv_dt, max_pos=W) for _ in range(B)]
    if block_size:
        nb = W // block_size
        pages = np.arange(B * nb)
        rng.shuffle(pages)
        for s in range(B):
            a.set_block_table(s, pages[s * nb:(s + 1) * nb])
    nan_rows = np.full((W, HKV * hd), 0x7FC1, dtype=np.uint16)   # quiet NaN in f16 and bf16
    for s in range(B):
        for l in range(L):
            a.write_cache(l, s, 0, W, torch.from_numpy(nan_rows.view(np.int16)).cuda(),
                          torch.from_numpy(nan_rows.view(np.int16)).cuda())
            peaky = rng.random(ctx[s]) < 0.01
            k, _ = random_kv_rows(rng, ctx[s], HKV * hd, kv_dt, peaky_rows=peaky)
            v, _ = random_kv_rows(rng, ctx[s], HKV * hd, kv_dt)
            kb, vb = k.view(np.uint16), v.view(np.uint16)
            a.write_cache(l, s, 0, ctx[s], torch.from_numpy(kb.view(np.int16)).cuda(),
                          torch.from_numpy(vb.view(np.int16)).cuda())
            seqs[s].k[l, :ctx[s]] = kb
            seqs[s].v[l, :ctx[s]] = vb
        a.set_state(s, ctx[s], 0)
        seqs[s].pos = ctx[s]
    worst = 0.0
    for _ in range(steps):
        q = rng.standard_normal((B, H * hd)).astype(np.float32)
        k = (rng.standard_normal((B, HKV * hd)) * 0.5).astype(np.float32)
        v = (rng.standard_normal((B, HKV * hd)) * 0.5).astype(np.float32)
        for l in range(L):
            out = torch.zeros((B, H * hd), dtype=torch.float32, device="cuda")
            a.decode(l, B, dev(q, kv_dt), dev(k, kv_dt), dev(v, kv_dt), out)
            a.sync()
            got = out.cpu().numpy()
            for s in range(B):
                want = seqs[s].step(l, O.round_act(q[s], kv_dt), O.round_act(k[s], kv_dt),
                                    O.round_act(v[s], kv_dt))
                worst = max(worst, rel_err(got[s].reshape(H, hd), want))
        a.advance(B)
        for s in seqs:
            s.advance()
    # Written rows bit-exact (the NaN fill beyond them is not the oracle's).
    for s, seq in enumerate(seqs):
        n = seq.pos
        for l in range(L):
            gk, gv, _, _ = a.read_cache(l, s, 0, n)
            ok, ov = oracle_cache(seq, l, kv_dt)
            assert np.array_equal(cache_bits(gk), cache_bits(ok[:n])), (s, l)
            assert np.array_equal(cache_bits(gv), cache_bits(ov[:n])), (s, l)
    a.close()
    return worst


@pytest.mark.parametrize("kv_dt", [O.F16, O.BF16])
@pytest.mark.parametrize("hd,rep", [(64, 1), (64, 2), (64, 4), (64, 8), (128, 1), (128, 2), (128, 4)])
def test_tma_decode_contiguous(kv_dt, hd, rep):
    worst = _session(kv_dt, hd, rep, 0, seed=11 + hd + rep, ctx=[1, 63, 64, 65, 700, 2047, 1283])
    assert worst <= TOL


@pytest.mark.parametrize("kv_dt", [O.F16, O.BF16])
@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("block_size", [64, 256])
def test_tma_decode_paged_shuffled(kv_dt, hd, block_size):
    worst = _session(kv_dt, hd, 2, block_size, seed=5 + block_size, ctx=[129, 2000, 511, 64])
    assert worst <= TOL


def test_config2_full_size_decode():
    """Config 2's decode shape at full size: 64 sequences, contexts U[256, 2048]
    (seed 1), 8x64 MHA, fp16 KV, one layer, four steps; the balanced grid's
    static and dynamic units and split items all occur at this size."""
    import torch
    rng = np.random.default_rng(1)
    B, H, HD, L = 64, 8, 64, 1
    ctx = rng.integers(256, 2049, size=B)
    W = 2176
    a = ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=H, window=W, max_seqs=B, kv_dtype="f16", act_dtype="f16",
                    out_dtype="f32", max_pos=W)
    seqs = [O.OracleSeq(L, H, H, HD, HD, W, O.F16, max_pos=W) for _ in range(B)]
    for s in range(B):
        n = int(ctx[s])
        k, _ = random_kv_rows(rng, n, H * HD, O.F16, peaky_rows=rng.random(n) < 0.01)
        v, _ = random_kv_rows(rng, n, H * HD, O.F16)
        a.write_cache(0, s, 0, n, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        seqs[s].k[0, :n] = k.view(np.uint16)
        seqs[s].v[0, :n] = v.view(np.uint16)
        a.set_state(s, n, 0)
        seqs[s].pos = n
    worst = 0.0
    for _ in range(4):
        q = rng.standard_normal((B, H * HD)).astype(np.float32)
        k = (rng.standard_normal((B, H * HD)) * 0.5).astype(np.float32)
        v = (rng.standard_normal((B, H * HD)) * 0.5).astype(np.float32)
        out = torch.zeros((B, H * HD), dtype=torch.float32, device="cuda")
        a.decode(0, B, dev(q, O.F16), dev(k, O.F16), dev(v, O.F16), out)
        a.sync()
        got = out.cpu().numpy()
        for s in range(B):
            want = seqs[s].step(0, O.round_act(q[s], O.F16), O.round_act(k[s], O.F16), O.round_act(v[s], O.F16))
            worst = max(worst, rel_err(got[s].reshape(H, HD), want))
        a.advance(B)
        for s in seqs:
            s.advance()
    assert worst <= TOL
    a.close()


def test_config4_geometry_long_context_paged():
    """Config 4's geometry at its full context: 32 768 cached tokens per
    sequence (8 sequences instead of 256), 8x128 MHA, fp16 KV ~ N(0,1) 0.25
    with 1 % of K rows x8, 64-slot pages in a shuffled block table (seed 3),
    two decode steps. Items hold 512 tiles here, so they span several static
    and dynamic units of the balanced grid."""
    import torch
    rng = np.random.default_rng(3)
    B, H, HD, CTX, BS = 8, 8, 128, 32768, 64
    W = CTX + 64
    a = ndattn.Attn(n_layers=1, n_heads=H, n_kv_heads=H, qk_head_dim=HD, v_head_dim=HD, window=W, max_seqs=B,
                    block_size=BS, kv_dtype="f16", act_dtype="f16", out_dtype="f32", max_pos=W)
    nb = W // BS
    pages = rng.permutation(B * nb)
    for s in range(B):
        a.set_block_table(s, pages[s * nb:(s + 1) * nb])
    seqs = [O.OracleSeq(1, H, H, HD, HD, W, O.F16, max_pos=W) for _ in range(B)]
    for s in range(B):
        k = rng.standard_normal((CTX, H * HD), dtype=np.float32) * 0.25
        k[rng.random(CTX) < 0.01] *= 8.0
        k = k.astype(np.float16)
        v = (rng.standard_normal((CTX, H * HD), dtype=np.float32) * 0.25).astype(np.float16)
        a.write_cache(0, s, 0, CTX, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        seqs[s].k[0, :CTX] = k.view(np.uint16)
        seqs[s].v[0, :CTX] = v.view(np.uint16)
        a.set_state(s, CTX, 0)
        seqs[s].pos = CTX
    worst = 0.0
    for _ in range(2):
        q = rng.standard_normal((B, H * HD)).astype(np.float32)
        k = (rng.standard_normal((B, H * HD)) * 0.25).astype(np.float32)
        v = (rng.standard_normal((B, H * HD)) * 0.25).astype(np.float32)
        out = torch.zeros((B, H * HD), dtype=torch.float32, device="cuda")
        a.decode(0, B, dev(q, O.F16), dev(k, O.F16), dev(v, O.F16), out)
        a.sync()
        got = out.cpu().numpy()
        for s in range(B):
            want = seqs[s].step(0, O.round_act(q[s], O.F16), O.round_act(k[s], O.F16), O.round_act(v[s], O.F16))
            worst = max(worst, rel_err(got[s].reshape(H, HD), want))
        a.advance(B)
        for s in seqs:
            s.advance()
    assert worst <= TOL
    for s in (0, B - 1):   # the appended rows, read back through the block table
        gk, gv, _, _ = a.read_cache(0, s, CTX, 2)
        ok, ov = oracle_cache(seqs[s], 0, O.F16)
        assert np.array_equal(cache_bits(gk), cache_bits(ok[CTX:CTX + 2]))
        assert np.array_equal(cache_bits(gv), cache_bits(ov[CTX:CTX + 2]))
    a.close()


@pytest.mark.parametrize("hd,rep,block_size", [(64, 1, 0), (64, 2, 0), (64, 1, 256), (128, 1, 128), (128, 2, 0), (64, 1, 64)])
def test_int8_balanced_decode(hd, rep, block_size):
    """int8 caches (the reference's own format, f32 activations) through the
    balanced kernel: KV-head counts whose scale rows are 16-byte multiples,
    so the scales arrive as TMA boxes beside the int8 rows (128-row tiles;
    64-row pages hold no whole tile and take the exact-grid kernel). Every slot is
    first poisoned with arbitrary int8 bytes and NaN scales; ragged contexts
    are then filled by prefill (K1 append + the balanced attend, outputs
    checked too) and decoded for two steps. Outputs within TOL of the oracle,
    KV bytes and scales bit-exact: rows past each item's end, read by the last
    box, must contribute nothing."""
    import torch
    rng = np.random.default_rng(101 + hd + rep + block_size)
    HKV = 8 if hd == 64 else 4
    H, L, W, B = HKV * rep, 2, 1536, 4
    ctx = [1, 63, 700, 1283]
    a = ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=HKV, qk_head_dim=hd, v_head_dim=hd, window=W, max_seqs=B,
                    kv_dtype="i8", act_dtype="f32", out_dtype="f32", block_size=block_size, max_pos=W)
    seqs = [O.OracleSeq(L, H, HKV, hd, hd, W, O.I8, max_pos=W) for _ in range(B)]
    if block_size:
        nb = W // block_size
        pages = rng.permutation(B * nb)
        for s in range(B):
            a.set_block_table(s, pages[s * nb:(s + 1) * nb])
    junk_k = torch.from_numpy(rng.integers(-128, 128, size=(W, HKV * hd), dtype=np.int8)).cuda()
    junk_v = torch.from_numpy(rng.integers(-128, 128, size=(W, HKV * hd), dtype=np.int8)).cuda()
    nan_sc = torch.full((W, HKV), float("nan"), dtype=torch.float32, device="cuda")
    for s in range(B):
        for l in range(L):
            a.write_cache(l, s, 0, W, junk_k, junk_v, nan_sc, nan_sc)
    worst = 0.0
    for s, n in enumerate(ctx):
        for l in range(L):
            q = rng.standard_normal((n, H * hd)).astype(np.float32)
            k = (rng.standard_normal((n, HKV * hd)) * 0.5).astype(np.float32)
            v = (rng.standard_normal((n, HKV * hd)) * 0.5).astype(np.float32)
            out = torch.zeros((n, H * hd), dtype=torch.float32, device="cuda")
            a.prefill(l, [n], dev(q, O.F32), dev(k, O.F32), dev(v, O.F32), out, seq_ids=[s])
            a.sync()
            got = out.cpu().numpy()
            for t in range(n):
                want = seqs[s].step(l, q[t], k[t], v[t], off=t)
                worst = max(worst, rel_err(got[t].reshape(H, hd), want))
        a.advance(1, seq_ids=[s], lens=[n])
        seqs[s].advance(n)
    for _ in range(2):
        q = rng.standard_normal((B, H * hd)).astype(np.float32)
        k = (rng.standard_normal((B, HKV * hd)) * 0.5).astype(np.float32)
        v = (rng.standard_normal((B, HKV * hd)) * 0.5).astype(np.float32)
        for l in range(L):
            out = torch.zeros((B, H * hd), dtype=torch.float32, device="cuda")
            a.decode(l, B, dev(q, O.F32), dev(k, O.F32), dev(v, O.F32), out)
            a.sync()
            got = out.cpu().numpy()
            for s in range(B):
                worst = max(worst, rel_err(got[s].reshape(H, hd), seqs[s].step(l, q[s], k[s], v[s])))
        a.advance(B)
        for s in seqs:
            s.advance()
    assert worst <= TOL, worst
    for s, seq in enumerate(seqs):
        n = seq.pos
        for l in range(L):
            gk, gv, gks, gvs = a.read_cache(l, s, 0, n)
            assert np.array_equal(gk, seq.k[l][:n]) and np.array_equal(gv, seq.v[l][:n]), (s, l)
            assert np.array_equal(gks.view(np.uint32), seq.ks[l][:n].view(np.uint32)), (s, l)
            assert np.array_equal(gvs.view(np.uint32), seq.vs[l][:n].view(np.uint32)), (s, l)
    a.close()
