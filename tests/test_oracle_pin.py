"""Pins the oracle restatement (oracle/nd_oracle.c) to the reference engine's
own attention code compiled from its sources (oracle/_ref/libndref.so):
kv_slot / set_sink over their whole input space of a window, RoPE tables,
int8 KV bytes and scales bit-exact, and attention outputs within 1e-5 of the
reference's fp32 result, over sessions that exercise sinks, ring wrap, GQA,
the per-head norm and the reference model's own 48/64 head geometry."""
import numpy as np
import pytest

import ndoracle as O

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) absent")


def test_kv_slot_and_sink_match_reference():
    r = O.ref()
    for window in (64, 65, 100, 384):
        for n_sink in (0, 1, 7, max(0, window - 64)):
            for p in range(0, 3 * window):
                assert O.kv_slot(window, n_sink, p) == r.ndref_kv_slot(window, n_sink, p)
        for n in range(0, window + 5):
            assert O.set_sink_cap(window, n) == r.ndref_set_sink(window, n)


@pytest.mark.parametrize("qk,theta", [(64, 10000.0), (48, 100000.0), (128, 10000.0)])
def test_rope_table_matches_reference(qk, theta):
    tab = O.rope_table(theta, qk, 40000)
    for pos in (0, 1, 2, 212, 383, 2047, 32768, 39999):
        cs, sn = O.ref_rope(theta, qk, pos)
        assert np.array_equal(tab[pos, :, 0], cs) and np.array_equal(tab[pos, :, 1], sn)


SESSIONS = [
    # H, HKV, QK, VD, window, layers, norm, prefix, sink, tokens
    (8, 8, 64, 64, 300, 1, False, 213, 213, 72),     # config 1 shape
    (12, 2, 48, 64, 384, 2, True, 40, 40, 30),       # the reference model's geometry
    (16, 4, 64, 64, 128, 1, False, 0, 0, 200),       # GQA 4:1, ring wraps (no sinks)
    (4, 1, 128, 128, 96, 1, True, 20, 20, 120),      # hd128, sinks + ring wrap
]


@pytest.mark.parametrize("H,HKV,QK,VD,W,L,norm,prefix,sink,tokens", SESSIONS)
def test_oracle_matches_reference_int8(H, HKV, QK, VD, W, L, norm, prefix, sink, tokens):
    rng = np.random.default_rng(7 + H + QK)
    ref = O.RefSeq(L, H, HKV, QK, VD, W, O.I8, max_pos=prefix + tokens + 1)
    orc = O.OracleSeq(L, H, HKV, QK, VD, W, O.I8, max_pos=prefix + tokens + 1)
    if norm:
        for l in range(L):
            qs = (rng.standard_normal(QK) * 0.1).astype(np.float32)
            ks = (rng.standard_normal(QK) * 0.1).astype(np.float32)
            ref.norms[l] = orc.norms[l] = (qs, ks)
    worst = 0.0
    for t in range(prefix + tokens):
        if t == prefix and sink:
            ref.set_sink(sink)
            orc.set_sink(sink)
        for l in range(L):
            q = (rng.standard_normal(H * QK) * 0.5).astype(np.float32)
            k = (rng.standard_normal(HKV * QK) * 0.5).astype(np.float32)
            v = (rng.standard_normal(HKV * VD) * 0.5).astype(np.float32)
            g = (rng.standard_normal(H * VD)).astype(np.float32) if t % 3 == 0 else None
            a = ref.step(l, q, k, v, g)
            b = orc.step(l, q, k, v, g)
            worst = max(worst, float(np.max(np.abs(a - b) / np.maximum(1.0, np.abs(b)))))
        ref.advance()
        orc.advance()
    assert np.array_equal(ref.k, orc.k) and np.array_equal(ref.v, orc.v)
    assert np.array_equal(ref.ks.view(np.uint32), orc.ks.view(np.uint32))
    assert np.array_equal(ref.vs.view(np.uint32), orc.vs.view(np.uint32))
    assert worst <= 1e-5, worst


def test_prefix_image_matches_reference():
    rng = np.random.default_rng(3)
    H, HKV, QK, VD, W, L = 8, 2, 64, 64, 300, 2
    ref = O.RefSeq(L, H, HKV, QK, VD, W, O.I8)
    mine = O.OracleSeq(L, H, HKV, QK, VD, W, O.I8)
    for t in range(213):
        for l in range(L):
            q = rng.standard_normal(H * QK).astype(np.float32)
            k = rng.standard_normal(HKV * QK).astype(np.float32)
            v = rng.standard_normal(HKV * VD).astype(np.float32)
            ref.step(l, q, k, v)
            mine.step(l, q, k, v)
        ref.advance()
        mine.advance()
    img, sink = ref.ref_prefix_image()
    mine.snapshot()
    assert sink == mine.n_sink == 213
    assert img == mine.prefix_image()


def test_quantiser_edge_rows():
    """Zero rows (scale 1), ties at .5 after division, tiny and huge values."""
    H, HKV, QK, VD, W = 2, 2, 64, 64, 128
    ref = O.RefSeq(1, H, HKV, QK, VD, W, O.I8)
    orc = O.OracleSeq(1, H, HKV, QK, VD, W, O.I8)
    rows = [np.zeros(QK), np.arange(QK) - 31.5, np.full(QK, 1e-30), (np.arange(QK) % 7 - 3) * 127.0 / 3.0,
            np.linspace(-1e4, 1e4, QK), np.where(np.arange(QK) % 2 == 0, 2.5, -0.5)]
    for i, r in enumerate(rows):
        k = np.concatenate([r, r[::-1]]).astype(np.float32)
        v = np.concatenate([r[::-1], r]).astype(np.float32)
        q = np.ones(H * QK, np.float32)
        ref.step(0, q, k, v)
        orc.step(0, q, k, v)
        ref.advance()
        orc.advance()
    assert np.array_equal(ref.k, orc.k) and np.array_equal(ref.v, orc.v)
    assert np.array_equal(ref.ks, orc.ks) and np.array_equal(ref.vs, orc.vs)
