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


@pytest.mark.parametrize("taps", [1, 2, 3, 4])
@pytest.mark.parametrize("dim", [48, 257])
def test_conv_taps_match_reference(taps, dim):
    """The QKV short causal convolution: the restatement against the
    reference's own tap_projection (nd_model.c:2361-2379), outputs and
    history bit for bit over positions 0.. (the ramp of min(taps, pos+1)
    taps, then every history slot reused), an odd width (the reference's
    two-column loop plus its tail) and signed zeros among the weights."""
    rng = np.random.default_rng(taps * 1000 + dim)
    w = (rng.standard_normal((taps, dim)) * 0.7).astype(np.float32)
    w[:, ::11] = 0.0
    w[:, 5::13] = -0.0
    h_ref = np.zeros((taps, dim), np.float32)
    h_mine = np.zeros((taps, dim), np.float32)
    for pos in range(3 * taps + 4):
        x = rng.standard_normal(dim).astype(np.float32)
        x[::7] = -0.0
        ref_row = x.copy()
        assert O.ref().ndref_tap(taps, pos, dim, w.ctypes.data, ref_row.ctypes.data, h_ref.ctypes.data) == 0
        out = np.zeros(dim, np.float32)
        assert O.orc().ndo_conv_taps(taps, pos, dim, w.ctypes.data, x.ctypes.data, h_mine.ctypes.data,
                                     out.ctypes.data) == 0
        assert np.array_equal(ref_row.view(np.uint32), out.view(np.uint32)), pos
        assert np.array_equal(h_ref.view(np.uint32), h_mine.view(np.uint32)), pos


def test_conv_taps_session_and_prefix_image_match_reference():
    """A session with 3 conv taps through both: the reference's tap_projection
    + attention and the restatement. Int8 KV bytes bit-exact, outputs within
    1e-5, and after a snapshot, a rewind and more tokens, the saved-prefix
    image (KV rows, scales, then q/k/v tap histories) byte for byte."""
    rng = np.random.default_rng(17)
    H, HKV, QK, VD, W, L, T = 8, 2, 64, 64, 160, 2, 3
    ref = O.RefSeq(L, H, HKV, QK, VD, W, O.I8, taps=T)
    mine = O.OracleSeq(L, H, HKV, QK, VD, W, O.I8, taps=T)
    for l in range(L):
        ws = [(rng.standard_normal((T, d)) * 0.6).astype(np.float32) for d in (H * QK, HKV * QK, HKV * VD)]
        ref.set_conv_taps(l, *ws)
        mine.set_conv_taps(l, *ws)
    worst = 0.0

    def tokens(n):
        nonlocal worst
        for _ in range(n):
            for l in range(L):
                q = (rng.standard_normal(H * QK) * 0.5).astype(np.float32)
                k = (rng.standard_normal(HKV * QK) * 0.5).astype(np.float32)
                v = (rng.standard_normal(HKV * VD) * 0.5).astype(np.float32)
                a, b = ref.step(l, q, k, v), mine.step(l, q, k, v)
                worst = max(worst, float(np.max(np.abs(a - b) / np.maximum(1.0, np.abs(b)))))
            ref.advance()
            mine.advance()

    tokens(40)
    ref.snapshot()
    mine.snapshot()
    tokens(5)
    ref.rewind()
    mine.rewind()
    tokens(3)
    assert np.array_equal(ref.k, mine.k) and np.array_equal(ref.v, mine.v)
    assert all(np.array_equal(a.view(np.uint32), b.view(np.uint32)) for a, b in zip(ref.hist, mine.hist))
    assert worst <= 1e-5, worst
    img, sink = ref.ref_prefix_image()
    mine.snapshot()
    assert sink == mine.n_sink and img == mine.prefix_image()


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
