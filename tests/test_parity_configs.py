"""Parity at the benchmarked shapes that the smaller session tests do not reach.

- Config 3 (batched causal prefill, GQA 16/4, hd 64, bf16) with 1024-token
  sequences: one call from position 0 gives every sequence 8 query tiles of
  128 tokens over up to 16 key tiles each, so the persistent kernel's
  longest-first item list, its diagonal tiles and its item boundaries all run
  as in the benchmark. A second call of ragged lengths then starts at 1024 over
  the cached prefix (diagonal tiles not aligned to the query tiles).
- Config 5 (shared-prefix serving) as a checked session: two schema prefixes
  (143 and 213 tokens, the reference firmware's two schemas, esp32/main/main.c
  208-253) prefilled into template sequences, saved (nd_model_prefix_save,
  nd_model.c:1531-1541), restored into 32 requests whose block tables map the
  template's whole prefix pages (nd_model_prefix_restore, nd_model.c:1543-1553),
  then a ragged suffix prefill of U[8, 64] tokens (seed 4) and 4 decode steps
  for all requests in each call (main.c:281-315). One request then switches
  schema (new block table, restore of the other prefix) and runs again.

Bars (harness.TOL): outputs within 1e-3 * max(1, |ref|) of the fp64 oracle,
caches bit-exact (paging resolved), the shared prefix pages untouched by the
requests' own writes.
"""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import ndattn
import ndoracle as O
from harness import TOL, cache_bits, dev, oracle_cache, rel_err

pytestmark = pytest.mark.gpu


def _out(n_tok, H, VD):
    import torch
    return torch.zeros((n_tok, H * VD), dtype=torch.float32, device="cuda")


def _oracle_calls(seqs, layer, jobs):
    """Runs the oracle for several sequences at once (its C calls release the
    GIL). jobs: per sequence index a list of (q, k, v, off) rows in token
    order; returns per sequence the stacked outputs."""
    def run(item):
        s, rows = item
        return s, np.stack([seqs[s].step(layer, q, k, v, off=off) for q, k, v, off in rows])
    with ThreadPoolExecutor(max_workers=min(16, len(jobs))) as ex:
        return dict(ex.map(run, jobs.items()))


def _check_caches(a, seqs, ids, kv_dt, L, W):
    for s, seq in zip(ids, seqs):
        for layer in range(L):
            k, v, _, _ = a.read_cache(layer, s, 0, W)
            ok, ov = oracle_cache(seq, layer, kv_dt)
            assert np.array_equal(cache_bits(k), cache_bits(ok)), (s, layer)
            assert np.array_equal(cache_bits(v), cache_bits(ov)), (s, layer)


def test_config3_full_length_prefill():
    H, HKV, D, W = 16, 4, 64, 1536
    lens1 = [1024] * 4
    lens2 = [300, 129, 1, 256]
    rng = np.random.default_rng(2)
    a = ndattn.Attn(n_layers=1, n_heads=H, n_kv_heads=HKV, qk_head_dim=D, v_head_dim=D, window=W,
                    max_seqs=len(lens1), kv_dtype="bf16", act_dtype="bf16", out_dtype="f32", max_pos=W)
    seqs = [O.OracleSeq(1, H, HKV, D, D, W, O.BF16, max_pos=W) for _ in lens1]
    worst = 0.0
    for lens in (lens1, lens2):
        T = sum(lens)
        q = O.round_act((rng.standard_normal((T, H * D)) * 0.5).astype(np.float32), O.BF16)
        k = O.round_act((rng.standard_normal((T, HKV * D)) * 0.5).astype(np.float32), O.BF16)
        v = O.round_act((rng.standard_normal((T, HKV * D)) * 0.5).astype(np.float32), O.BF16)
        out = _out(T, H, D)
        a.prefill(0, lens, dev(q, O.BF16), dev(k, O.BF16), dev(v, O.BF16), out)
        a.sync()
        got = out.cpu().numpy()
        cu = np.concatenate([[0], np.cumsum(lens)])
        jobs = {s: [(q[cu[s] + t], k[cu[s] + t], v[cu[s] + t], t) for t in range(n)] for s, n in enumerate(lens)}
        want = _oracle_calls(seqs, 0, jobs)
        for s, n in enumerate(lens):
            worst = max(worst, rel_err(got[cu[s]:cu[s] + n].reshape(n, H, D), want[s]))
        a.advance(len(lens), lens=lens)
        for s, n in zip(seqs, lens):
            s.advance(n)
        assert worst <= TOL, worst
    _check_caches(a, seqs, range(len(seqs)), O.BF16, 1, W)
    a.close()


def test_config5_shared_prefix_session_two_schemas():
    import torch
    H = HKV = 8
    D, L, BS = 64, 2, 64
    prefixes = (143, 213)
    n_req, dec_steps = 32, 4
    W = (max(prefixes) + 64 + dec_steps + 1 + BS - 1) // BS * BS + BS     # room for the schema switch
    nb = W // BS
    rng = np.random.default_rng(4)
    tpl = [n_req, n_req + 1]                                              # template sequence ids
    n_blocks = (n_req + 2) * nb
    a = ndattn.Attn(n_layers=L, n_heads=H, n_kv_heads=HKV, qk_head_dim=D, v_head_dim=D, window=W,
                    max_seqs=n_req + 2, block_size=BS, n_blocks=n_blocks, kv_dtype="f16", act_dtype="f16",
                    out_dtype="f32", max_pos=W)
    mk = lambda: O.OracleSeq(L, H, HKV, D, D, W, O.F16, max_pos=W)  # noqa: E731
    tpl_pages = [np.arange(i * nb, (i + 1) * nb) for i in range(2)]
    for i in range(2):
        a.set_block_table(tpl[i], tpl_pages[i])

    def x(n, width):
        return O.round_act((rng.standard_normal((n, width)) * 0.5).astype(np.float32), O.F16)

    # Template prefills: both schemas in one call per layer.
    tseq = [mk(), mk()]
    T = sum(prefixes)
    cu = [0, prefixes[0]]
    worst = 0.0
    for layer in range(L):
        q, k, v = x(T, H * D), x(T, HKV * D), x(T, HKV * D)
        out = _out(T, H, D)
        a.prefill(layer, list(prefixes), dev(q, O.F16), dev(k, O.F16), dev(v, O.F16), out, seq_ids=tpl)
        a.sync()
        got = out.cpu().numpy()
        jobs = {i: [(q[cu[i] + t], k[cu[i] + t], v[cu[i] + t], t) for t in range(p)] for i, p in enumerate(prefixes)}
        want = _oracle_calls(tseq, layer, jobs)
        for i, p in enumerate(prefixes):
            worst = max(worst, rel_err(got[cu[i]:cu[i] + p].reshape(p, H, D), want[i]))
    a.advance(2, seq_ids=tpl, lens=list(prefixes))
    saved, osaved = [], []
    for i in range(2):
        tseq[i].advance(prefixes[i])
        a.snapshot(tpl[i])
        tseq[i].snapshot()
        saved.append(a.prefix_save(tpl[i]))
        assert saved[-1] is not None
        osaved.append(tseq[i].prefix_save())
        img, ppos, _ = saved[-1].read()
        assert ppos == prefixes[i]
        assert img.tobytes() == tseq[i].prefix_image()

    # Requests: even ones on the 143-token schema, odd ones on the 213-token one.
    schema = [r % 2 for r in range(n_req)]

    def table(r, sch):
        shared = prefixes[sch] // BS                     # whole prefix pages, shared with the template
        own = (2 + r) * nb + np.arange(nb - shared)
        return np.concatenate([tpl_pages[sch][:shared], own])

    rseq = []
    for r in range(n_req):
        a.set_block_table(r, table(r, schema[r]))
        a.prefix_restore(r, saved[schema[r]])
        s = mk()
        s.prefix_restore(osaved[schema[r]])
        rseq.append(s)
        assert a.state(r) == (s.pos, s.n_sink)

    def serve(ids, suf):
        nonlocal worst
        Ts = int(sum(suf))
        cs = np.concatenate([[0], np.cumsum(suf)])
        for layer in range(L):                       # ragged suffix prefill, all requests in one call
            q, k, v = x(Ts, H * D), x(Ts, HKV * D), x(Ts, HKV * D)
            out = _out(Ts, H, D)
            a.prefill(layer, [int(n) for n in suf], dev(q, O.F16), dev(k, O.F16), dev(v, O.F16), out, seq_ids=ids)
            a.sync()
            got = out.cpu().numpy()
            jobs = {j: [(q[cs[j] + t], k[cs[j] + t], v[cs[j] + t], t) for t in range(int(n))]
                    for j, n in enumerate(suf)}
            want = _oracle_calls([rseq[r] for r in ids], layer, jobs)
            for j, n in enumerate(suf):
                worst = max(worst, rel_err(got[cs[j]:cs[j] + n].reshape(int(n), H, D), want[j]))
        a.advance(len(ids), seq_ids=ids, lens=[int(n) for n in suf])
        for r, n in zip(ids, suf):
            rseq[r].advance(int(n))
        for _ in range(dec_steps):                   # decode steps, all requests in each call
            for layer in range(L):
                q, k, v = x(len(ids), H * D), x(len(ids), HKV * D), x(len(ids), HKV * D)
                out = _out(len(ids), H, D)
                a.decode(layer, len(ids), dev(q, O.F16), dev(k, O.F16), dev(v, O.F16), out, seq_ids=ids)
                a.sync()
                got = out.cpu().numpy()
                want = _oracle_calls([rseq[r] for r in ids], layer, {j: [(q[j], k[j], v[j], 0)]
                                                                     for j in range(len(ids))})
                for j in range(len(ids)):
                    worst = max(worst, rel_err(got[j].reshape(1, H, D), want[j]))
            a.advance(len(ids), seq_ids=ids)
            for r in ids:
                rseq[r].advance()

    ids = list(range(n_req))
    serve(ids, rng.integers(8, 65, size=n_req))
    assert worst <= TOL, worst
    _check_caches(a, rseq, ids, O.F16, L, W)
    _check_caches(a, tseq, tpl, O.F16, L, W)         # the shared prefix pages still hold the prefixes

    # Schema switch (nd_ptest's pattern): request 0 moves to the other prefix.
    r0 = 0
    new = 1 - schema[r0]
    a.set_block_table(r0, table(r0, new))
    a.prefix_restore(r0, saved[new])
    rseq[r0] = mk()
    rseq[r0].prefix_restore(osaved[new])
    assert a.state(r0) == (prefixes[new], rseq[r0].n_sink)
    serve([r0, 1], np.array([37, 12]))
    assert worst <= TOL, worst
    _check_caches(a, [rseq[r0], rseq[1]], [r0, 1], O.F16, L, W)
    _check_caches(a, tseq, tpl, O.F16, L, W)
    for p in saved:
        p.free()
    a.close()
    del torch
