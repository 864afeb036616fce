"""nd_attn_decode_shared: decode of requests that all begin with one schema
prefix, with the prefix rows read once per CTA from the template sequence.

Each session: a template sequence prefills the prefix, snapshots and saves it
(nd_model_snapshot / nd_model_prefix_save, engine/src/nd_model.c:1395-1541);
every request restores it (nd_model_prefix_restore, nd_model.c:1543-1553), as
the firmware does per request (esp32/main/main.c:281-315), prefills a ragged
suffix, then decodes several steps through nd_attn_decode_shared. Paged caches
map the template's whole prefix pages into every request's block table;
contiguous caches hold a restored copy per request. Every output is compared
with its own oracle sequence (harness.TOL), the caches bit for bit, and the
template's caches are checked untouched.

Covered: f16 MHA 8x64 over two schemas in one handle (config 5's shape, paged)
on both kernels, int8 with GQA 4:1 plus head norms and gates, bf16 at head dim
128 with GQA 2:1 (the lane-map kernel), and f32 at the reference model's
12/2 x 48/64 geometry. The host refusals (prefix rows not written, a request
inside the prefix, a ring that wraps) launch nothing and leave the session
usable.
"""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import ndattn
import ndoracle as O
from harness import TOL, cache_bits, dev, oracle_cache, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _force_kernel(monkeypatch):
    """The library takes its regular decode for calls this small; the tests
    force the shared-prefix kernels (variant 2 where built, else variant 1)."""
    monkeypatch.setenv("ND_ATTN_SHARED_VARIANT", "2")


def _run_oracle(seqs, layer, rows, gate):
    """One oracle step per listed sequence (C calls release the GIL)."""
    def run(i):
        q, k, v = rows[0][i], rows[1][i], rows[2][i]
        return seqs[i].step(layer, q, k, v, None if gate is None else gate[i], off=0)
    with ThreadPoolExecutor(max_workers=min(16, len(seqs))) as ex:
        return list(ex.map(run, range(len(seqs))))


def _check_caches(a, seqs, ids, kv_dt, L, W):
    for s, seq in zip(ids, seqs):
        for layer in range(L):
            k, v, ks, vs = a.read_cache(layer, s, 0, W)
            ok, ov = oracle_cache(seq, layer, kv_dt)
            assert np.array_equal(cache_bits(k), cache_bits(ok)), (s, layer)
            assert np.array_equal(cache_bits(v), cache_bits(ov)), (s, layer)
            if kv_dt == O.I8:
                assert np.array_equal(ks, seq.ks[layer]) and np.array_equal(vs, seq.vs[layer]), (s, layer)


def _session(kv_dt, act_dt, H, HKV, QK, VD, prefixes, n_req, dec_steps, seed, block_size=0, norm=False,
             gate=False, L=2):
    """Runs the session described in the module docstring; returns the worst
    relative error of the shared-prefix decode outputs."""
    import torch
    rng = np.random.default_rng(seed)
    BS = block_size
    W = max(prefixes) + 64 + dec_steps + 1
    W = (W + 63) // 64 * 64 + (BS or 64)
    n_tpl = len(prefixes)
    tpl = [n_req + i for i in range(n_tpl)]
    kw = dict(n_layers=L, n_heads=H, n_kv_heads=HKV, qk_head_dim=QK, v_head_dim=VD, window=W,
              max_seqs=n_req + n_tpl, kv_dtype=kv_dt, act_dtype=act_dt, out_dtype="f32", max_pos=W)
    nb = W // BS if BS else 0
    if BS:
        kw.update(block_size=BS, n_blocks=(n_req + n_tpl) * nb)
    a = ndattn.Attn(**kw)
    mk = lambda: O.OracleSeq(L, H, HKV, QK, VD, W, kv_dt, max_pos=W)  # noqa: E731
    tpl_pages = [np.arange(i * nb, (i + 1) * nb) for i in range(n_tpl)] if BS else None
    if BS:
        for i in range(n_tpl):
            a.set_block_table(tpl[i], tpl_pages[i])
    norms = []
    if norm:
        for layer in range(L):
            qs = (rng.standard_normal(QK) * 0.1).astype(np.float32)
            ks = (rng.standard_normal(QK) * 0.1).astype(np.float32)
            a.set_head_norm(layer, qs, ks)
            norms.append((qs, ks))

    def new_seq():
        s = mk()
        for layer, nn in enumerate(norms):
            s.norms[layer] = nn
        return s

    def x(n, width, scale=0.5):
        return O.round_act((rng.standard_normal((n, width)) * scale).astype(np.float32), act_dt)

    def out(n):
        return torch.zeros((n, H * VD), dtype=torch.float32, device="cuda")

    # Templates: prefill each schema prefix, snapshot, save.
    tseq = [new_seq() for _ in range(n_tpl)]
    for i, p in enumerate(prefixes):
        for layer in range(L):
            q, k, v = x(p, H * QK), x(p, HKV * QK), x(p, HKV * VD)
            a.prefill(layer, [p], dev(q, act_dt), dev(k, act_dt), dev(v, act_dt), out(p), seq_ids=[tpl[i]])
            for t in range(p):
                tseq[i].step(layer, q[t], k[t], v[t], off=t)
        a.advance(1, seq_ids=[tpl[i]], lens=[p])
        tseq[i].advance(p)
    saved, osaved = [], []
    for i in range(n_tpl):
        a.snapshot(tpl[i])
        tseq[i].snapshot()
        saved.append(a.prefix_save(tpl[i]))
        osaved.append(tseq[i].prefix_save())

    # Requests: request r on schema r % n_tpl.
    schema = [r % n_tpl for r in range(n_req)]
    rseq = []
    for r in range(n_req):
        if BS:
            shared = prefixes[schema[r]] // BS
            own = (n_tpl + r) * nb + np.arange(nb - shared)
            a.set_block_table(r, np.concatenate([tpl_pages[schema[r]][:shared], own]))
        a.prefix_restore(r, saved[schema[r]])
        s = new_seq()
        s.prefix_restore(osaved[schema[r]])
        rseq.append(s)

    # Ragged suffix prefill of every request in one call per layer.
    suf = [int(n) for n in rng.integers(1, 40, size=n_req)]
    T = sum(suf)
    cs = np.concatenate([[0], np.cumsum(suf)])
    for layer in range(L):
        q, k, v = x(T, H * QK), x(T, HKV * QK), x(T, HKV * VD)
        a.prefill(layer, suf, dev(q, act_dt), dev(k, act_dt), dev(v, act_dt), out(T))
        for r in range(n_req):
            for t in range(suf[r]):
                rseq[r].step(layer, q[cs[r] + t], k[cs[r] + t], v[cs[r] + t], off=t)
    a.advance(n_req, lens=suf)
    for r in range(n_req):
        rseq[r].advance(suf[r])

    # Decode steps through the shared-prefix entry point, one call per schema.
    worst = 0.0
    groups = [[r for r in range(n_req) if schema[r] == i] for i in range(n_tpl)]
    for _ in range(dec_steps):
        for layer in range(L):
            for i, ids in enumerate(groups):
                n = len(ids)
                q, k, v = x(n, H * QK), x(n, HKV * QK), x(n, HKV * VD)
                g = x(n, H * VD, 1.0) if gate else None
                o = out(n)
                a.decode_shared(layer, n, tpl[i], prefixes[i], dev(q, act_dt), dev(k, act_dt), dev(v, act_dt), o,
                                gate=None if g is None else dev(g, act_dt), seq_ids=ids)
                a.sync()
                got = o.cpu().numpy()
                want = _run_oracle([rseq[r] for r in ids], layer, (q, k, v), g)
                for j in range(n):
                    worst = max(worst, rel_err(got[j].reshape(H, VD), want[j]))
        a.advance(n_req)
        for s in rseq:
            s.advance()
    _check_caches(a, rseq, range(n_req), kv_dt, L, W)
    _check_caches(a, tseq, tpl, kv_dt, L, W)        # the templates' rows (shared pages) untouched
    for p in saved:
        p.free()
    a.close()
    return worst


@pytest.mark.parametrize("variant", ["2", "1"])
def test_shared_prefix_f16_mha_paged_two_schemas(variant, monkeypatch):
    """Config 5's head shape (8x64 MHA, f16, 64-slot pages) with the 143- and
    213-token schemas in one handle, on both kernels: one lane per query row
    over the prefix (variant 2, the default at head dims up to 64) and the lane
    map throughout (variant 1, four tokens per warp)."""
    monkeypatch.setenv("ND_ATTN_SHARED_VARIANT", variant)
    worst = _session(O.F16, O.F16, 8, 8, 64, 64, (143, 213), n_req=40, dec_steps=3, seed=4, block_size=64)
    assert worst <= TOL, worst


def test_shared_prefix_int8_gqa4_norm_gate():
    """int8 caches (the reference's format), GQA 4:1, head norms and gates,
    contiguous cache."""
    worst = _session(O.I8, O.F32, 8, 2, 64, 64, (100,), n_req=12, dec_steps=3, seed=7, norm=True, gate=True)
    assert worst <= TOL, worst


def test_shared_prefix_bf16_hd128_gqa2():
    """bf16 at head dim 128, GQA 2:1, paged: the lane-map kernel with two
    tokens of two query rows per warp."""
    worst = _session(O.BF16, O.BF16, 8, 4, 128, 128, (150,), n_req=10, dec_steps=2, seed=8, block_size=64)
    assert worst <= TOL, worst


def test_shared_prefix_f32_reference_geometry():
    """The reference model's attention geometry (12/2 heads, qk 48, v 64),
    f32 caches, norms and gates."""
    worst = _session(O.F32, O.F32, 12, 2, 48, 64, (77,), n_req=9, dec_steps=2, seed=9, norm=True, gate=True)
    assert worst <= TOL, worst


def test_shared_prefix_refusals_launch_nothing():
    import torch
    H = HKV = 4
    D, W = 64, 128
    a = ndattn.Attn(n_layers=1, n_heads=H, n_kv_heads=HKV, qk_head_dim=D, v_head_dim=D, window=W, max_seqs=4,
                    kv_dtype="f16", act_dtype="f16", out_dtype="f32", max_pos=4 * W)
    q = torch.zeros((2, H * D), dtype=torch.float16, device="cuda")
    kv = torch.zeros((2, HKV * D), dtype=torch.float16, device="cuda")
    o = torch.zeros((2, H * D), dtype=torch.float32, device="cuda")
    a.set_state(2, 50, 0)                      # the prefix sequence: 50 rows written
    a.set_state(0, 60, 0)

    def refused(pos1, prefix_rows):
        a.set_state(1, pos1, 0)
        before = a.launches
        with pytest.raises(ndattn.NdAttnError) as e:
            a.decode_shared(0, 2, 2, prefix_rows, q, kv, kv, o)
        assert e.value.code == ndattn.ERR_RANGE
        assert a.launches == before

    refused(70, 51)          # more prefix rows than the prefix sequence holds
    refused(40, 50)          # a request still inside the prefix
    refused(W + 5, 50)       # a position that wraps the ring
    a.set_state(1, 70, 0)
    a.decode_shared(0, 2, 2, 50, q, kv, kv, o)      # the handle still works
    a.sync()
    assert np.isfinite(o.cpu().numpy()).all()
    a.close()
